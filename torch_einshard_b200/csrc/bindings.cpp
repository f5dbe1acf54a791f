// Torch bindings of the native einshard kernels (module torch_einshard_b200._C).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>

#include "comm.h"
#include "conv.h"
#include "copy.h"
#include "fft.h"
#include "gemm.h"
#include "act.h"
#include "gemm_ar.h"
#include "gemm_nvls.h"
#include "nvls.h"
#include "symm.h"
#include "tma_desc.h"

#include <memory>
#include <vector>

namespace es {
int* noalloc_status_word();  // noalloc_gemm.cu
}

namespace {

// Number of native kernel launches issued through these bindings (all devices).
std::atomic<long long> g_launches{0};
// -1: heuristic; 0/1: force the 1-SM / 2-SM GEMM kernel (tests, tuning)
int g_pair_mode = -1;
int g_group_m = 0;  // raster group override (0: kernel default)
int g_split = 0;    // wide-kernel cluster split mode (tuning)
int g_sleep_ns = 0;  // wide-kernel epilogue back-off (tuning)
int g_small_persistent = 1;  // 1-SM GEMM and conv grids (tuning)
uint64_t g_wait_timeout_ns = 4000000000ull;  // bound of device waits on peers (EINSHARD_WAIT_TIMEOUT_US)
int g_streamk = -1;  // stream-K on the wide kernel: -1 the partial last wave of long-K GEMMs (default), 1 every tile, 0 never
int g_persistent = -1;  // wide-kernel grid: 0 one pair tile per cluster, 1 persistent, -1 by K (default)
unsigned long long* g_prof = nullptr;  // wide-kernel wait counters (tuning), device pointer or null

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16:
      return es::kDtypeBF16;
    case at::kHalf:
      return es::kDtypeF16;
    case at::kFloat:
      return es::kDtypeF32;
    default:
      TORCH_CHECK(false, "einshard native: unsupported dtype ", t);
  }
}

int num_sms(int device) {
  static int cache[64] = {0};
  if (!cache[device]) {
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, device);
    cache[device] = prop.multiProcessorCount;
  }
  return cache[device];
}

// Fill operand layout fields from a [batch, rows, K] (A) or [batch, K, cols] (B) view.
void operand_layout(const at::Tensor& t, bool is_a, int& mn, long long& ld, long long& bstride) {
  // A: dims (M, K); B: dims (K, N).  "mn" means the non-K dim is contiguous.
  const int kdim = is_a ? 2 : 1;
  const int xdim = is_a ? 1 : 2;
  if (t.stride(kdim) == 1 && (t.size(xdim) == 1 || t.stride(xdim) != 1 || t.size(kdim) > 1)) {
    mn = 0;
    ld = t.size(xdim) == 1 ? std::max<long long>(t.stride(xdim), t.size(kdim)) : t.stride(xdim);
  } else {
    TORCH_CHECK(t.stride(xdim) == 1, "einshard native gemm: operand needs a unit stride in its last two dims");
    mn = 1;
    ld = t.size(kdim) == 1 ? std::max<long long>(t.stride(kdim), t.size(xdim)) : t.stride(kdim);
  }
  bstride = t.stride(0);
}

es::GemmArgs gemm_args(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t act, const at::Tensor& err);

void run_gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t act, const at::Tensor& err) {
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g = gemm_args(a, b, out, act, err);
  // stream-K adds fp32 partial tiles in arrival order: skipped when torch asks for deterministic algorithms
  es::StreamKPlan plan;
  if ((g.pair < 0 || g_streamk > 0) && !at::globalContext().deterministicAlgorithms() &&
      es::gemm_streamk_plan(g, g_streamk, &plan)) {
    // fp32 workspace from the caching allocator (the stream orders its reuse)
    at::Tensor ws = at::empty({es::gemm_streamk_ws_elems(plan)}, a.options().dtype(at::kFloat));
    const int rc = es::gemm_launch_streamk(g, plan, ws.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(rc == 0, "einshard native gemm: stream-K launch failed (", rc, ")");
    // whole tiles (when any), the tail and the finishing pass
    g_launches.fetch_add(plan.sk_first > 0 ? 3 : 2, std::memory_order_relaxed);
    return;
  }
  const int rc = es::gemm_launch(g, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard native gemm: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// Operand fields of a GEMM (the output fields are filled by the caller).
es::GemmArgs gemm_operand_args(const at::Tensor& a, const at::Tensor& b, int64_t act, const at::Tensor& err) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "einshard native gemm: CUDA tensors required");
  TORCH_CHECK(a.dim() == 3 && b.dim() == 3, "einshard native gemm: 3-D operands required");
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "einshard native gemm: operand dtypes differ");
  TORCH_CHECK(a.size(0) == b.size(0) && a.size(2) == b.size(1), "einshard native gemm: shape mismatch");
  es::GemmArgs g;
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.dtype = dtype_code(a.scalar_type());
  TORCH_CHECK(g.dtype != es::kDtypeF32, "einshard native gemm: bf16/fp16 operands required");
  g.batch = a.size(0);
  g.M = a.size(1);
  g.K = a.size(2);
  g.N = b.size(2);
  operand_layout(a, true, g.a_mn, g.lda, g.a_batch_stride);
  operand_layout(b, false, g.b_mn, g.ldb, g.b_batch_stride);
  g.act = static_cast<int>(act);
  g.err = err.data_ptr<int>();
  g.num_sms = num_sms(a.get_device());
  g.pair = g_pair_mode;
  g.group_m = g_group_m;
  g.split = g_split;
  g.prof = g_prof;
  g.sleep_ns = g_sleep_ns;
  g.persistent = g_persistent;
  g.small_persistent = g_small_persistent;
  return g;
}

es::GemmArgs gemm_args(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t act, const at::Tensor& err) {
  TORCH_CHECK(out.is_cuda() && out.dim() == 3, "einshard native gemm: 3-D CUDA output required");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == a.size(1) && out.size(2) == b.size(2),
              "einshard native gemm: output shape mismatch");
  TORCH_CHECK(out.stride(2) == 1, "einshard native gemm: output must be row-major");
  es::GemmArgs g = gemm_operand_args(a, b, act, err);
  g.C = out.data_ptr();
  g.out_dtype = dtype_code(out.scalar_type());
  g.ldc = out.stride(1);
  g.c_batch_stride = out.stride(0);
  const char* why = es::check_gemm_args(g);
  TORCH_CHECK(why == nullptr, "einshard native gemm: ", why ? why : "");
  return g;
}

at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, int64_t out_dtype, int64_t act, const at::Tensor& err) {
  at::ScalarType ot = out_dtype == es::kDtypeF32 ? at::kFloat : (out_dtype == es::kDtypeF16 ? at::kHalf : at::kBFloat16);
  at::Tensor out = at::empty({a.size(0), a.size(1), b.size(2)}, a.options().dtype(ot));
  run_gemm(a, b, out, act, err);
  return out;
}

void gemm_out(const at::Tensor& a, const at::Tensor& b, at::Tensor out, int64_t act, const at::Tensor& err) {
  run_gemm(a, b, out, act, err);
}

int act_dtype(const at::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf, "einshard silu: bf16 or fp16");
  return t.scalar_type() == at::kBFloat16 ? 0 : 1;
}

// (silu(a @ b), a @ b): one pass over the accumulator on the wide kernel, else
// the GEMM followed by the elementwise activation.
std::vector<at::Tensor> gemm_silu(const at::Tensor& a, const at::Tensor& b, const at::Tensor& err) {
  at::Tensor out = at::empty({a.size(0), a.size(1), b.size(2)}, a.options());
  at::Tensor pre = at::empty_like(out);
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g = gemm_args(a, b, out, es::kActSiluDual, err);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int rc = es::gemm_launch_silu_dual(g, pre.data_ptr(), pre.stride(1), pre.stride(0), stream);
  if (rc == 0) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return {out, pre};
  }
  TORCH_CHECK(rc == static_cast<int>(cudaErrorNotSupported), "einshard gemm+silu: launch failed (", rc, ")");
  run_gemm(a, b, pre, 0, err);
  rc = es::silu_forward(pre.data_ptr(), out.data_ptr(), out.numel(), act_dtype(out), num_sms(a.get_device()), stream);
  TORCH_CHECK(rc == 0, "einshard silu: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return {out, pre};
}

at::Tensor silu_forward(const at::Tensor& h) {
  TORCH_CHECK(h.is_cuda() && h.is_contiguous(), "einshard silu: contiguous CUDA tensor");
  at::Tensor out = at::empty_like(h);
  const c10::cuda::CUDAGuard guard(h.device());
  const int rc = es::silu_forward(h.data_ptr(), out.data_ptr(), h.numel(), act_dtype(h), num_sms(h.get_device()),
                                  at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard silu: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return out;
}

// grad * silu'(h)
at::Tensor silu_backward(const at::Tensor& grad, const at::Tensor& h) {
  TORCH_CHECK(h.is_cuda() && h.is_contiguous() && grad.is_contiguous() && grad.sizes() == h.sizes() &&
                  grad.scalar_type() == h.scalar_type(),
              "einshard silu backward: contiguous tensors of one shape and dtype");
  at::Tensor out = at::empty_like(h);
  const c10::cuda::CUDAGuard guard(h.device());
  const int rc = es::silu_backward(grad.data_ptr(), h.data_ptr(), out.data_ptr(), h.numel(), act_dtype(h),
                                   num_sms(h.get_device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard silu backward: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return out;
}


// ------------------------------------------------------------------ communicators

struct HostComm {
  int rank = 0, size = 1, device = 0;
  es::SymmHeap heap;         // cuMem allocations of every rank + multicast object (symm.h)
  void* local = nullptr;     // this rank's heap: [flags][data]
  std::vector<void*> bases;  // per rank: heap base (peer-mapped for peers)
  void* mc = nullptr;        // multicast view of the heap (nullptr without NVLS)
  size_t data_bytes = 0;
  int epoch = 0;
  uint32_t bar = 0;
  uint32_t arrive = 0;
  int nvls_epoch = 0;        // collectives issued on the NVLS counters
  int nvls_blocks = 0;       // fixed block count of every NVLS collective on this heap
  int tile_epoch = 0;        // fused GEMM + all-reduce calls (per-unit counters)
  bool open = false;
};

std::vector<std::unique_ptr<HostComm>> g_comms;

HostComm& comm_ref(int64_t id) {
  TORCH_CHECK(id >= 0 && id < (int64_t)g_comms.size() && g_comms[id], "einshard comm: bad communicator id");
  return *g_comms[id];
}

bool symm_multicast_supported(int64_t device) { return es::symm_multicast_supported(static_cast<int>(device)); }

// Phase 1 of creating a communicator over a symmetric heap (symm.h): allocate
// this rank's memory (and, on rank 0, the multicast object) and open the
// socket peers fetch the descriptors from.  Returns (id, error message).
py::tuple symm_prepare(int64_t data_bytes, int64_t device, const std::string& tag, int64_t rank, int64_t size,
                       bool want_mc, int64_t nvls_blocks) {
  TORCH_CHECK(size >= 1 && size <= es::kMaxRanks, "einshard comm: 1 to 8 ranks");
  TORCH_CHECK(nvls_blocks >= 1 && nvls_blocks <= es::kNvlsMaxBlocks, "einshard comm: NVLS block count");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  auto hc = std::make_unique<HostComm>();
  hc->rank = static_cast<int>(rank);
  hc->size = static_cast<int>(size);
  hc->device = static_cast<int>(device);
  hc->nvls_blocks = static_cast<int>(nvls_blocks);
  const std::string err = es::symm_prepare(hc->heap, es::kFlagBytes + static_cast<size_t>(data_bytes),
                                           static_cast<int>(device), tag, hc->rank, hc->size, want_mc);
  g_comms.push_back(std::move(hc));
  return py::make_tuple(static_cast<int64_t>(g_comms.size() - 1), err);
}

// Phase 2: fetch peers' descriptors, map every rank's memory, join the multicast team.
std::string symm_exchange(int64_t id, double timeout_s) {
  HostComm& hc = comm_ref(id);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(hc.device));
  return es::symm_exchange(hc.heap, timeout_s);
}

// Phase 3 (after every rank joined the team): bind this rank's memory to the multicast object.
std::string symm_bind(int64_t id) {
  HostComm& hc = comm_ref(id);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(hc.device));
  return es::symm_bind(hc.heap);
}

// Phase 4: map the multicast object, zero this rank's flag words, open the communicator.
std::string symm_finish(int64_t id) {
  HostComm& hc = comm_ref(id);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(hc.device));
  std::string err = es::symm_map_mc(hc.heap);
  if (!err.empty()) return err;
  const es::SymmHeap& h = hc.heap;
  hc.bases.assign(hc.size, nullptr);
  for (int p = 0; p < hc.size; ++p) hc.bases[p] = reinterpret_cast<void*>(h.uc_base + p * h.bytes);
  hc.local = hc.bases[hc.rank];
  hc.mc = h.mc_mapped ? reinterpret_cast<void*>(h.mc_base) : nullptr;
  hc.data_bytes = h.bytes - es::kFlagBytes;
  if (cudaMemset(hc.local, 0, es::kFlagBytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
    return "zeroing the flag words failed";
  hc.open = true;
  return "";
}

// Unmap and free (after a device synchronisation and a barrier of every rank).
void comm_destroy(int64_t id) {
  HostComm& hc = comm_ref(id);
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(hc.device));
  cudaDeviceSynchronize();
  es::symm_destroy(hc.heap);
  g_comms[id].reset();
}

bool comm_has_multicast(int64_t id) { return comm_ref(id).mc != nullptr; }

es::CommDev make_dev(HostComm& hc, const at::Tensor& err, int nblocks, int nbarriers) {
  es::CommDev d;
  d.rank = hc.rank;
  d.size = hc.size;
  for (int p = 0; p < es::kMaxRanks; ++p) {
    d.flags[p] = p < hc.size ? reinterpret_cast<uint64_t>(hc.bases[p]) : 0;
    d.data[p] = p < hc.size ? reinterpret_cast<uint64_t>(hc.bases[p]) + es::kFlagBytes : 0;
  }
  d.epoch = ++hc.epoch;
  d.bar_base = hc.bar;
  d.arrive_base = 0;
  d.err = err.data_ptr<int>();
  d.timeout_ns = g_wait_timeout_ns;
  hc.bar += static_cast<uint32_t>(nblocks * nbarriers);
  return d;
}

int es_dtype(const at::Tensor& t) {
  return t.scalar_type() == at::kBFloat16 ? 0 : t.scalar_type() == at::kHalf ? 1 : 2;
}

void comm_all_reduce(int64_t id, at::Tensor buf, double scale, int64_t nblocks, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open && buf.is_cuda() && buf.is_contiguous(), "einshard comm all_reduce: bad arguments");
  TORCH_CHECK(buf.scalar_type() == at::kBFloat16 || buf.scalar_type() == at::kHalf || buf.scalar_type() == at::kFloat,
              "einshard comm all_reduce: dtype");
  const int64_t bytes = buf.numel() * buf.element_size();
  const int64_t per = (bytes / 16 + hc.size - 1) / hc.size * 16;
  TORCH_CHECK(bytes % 16 == 0 && (size_t)(bytes + per) <= hc.data_bytes, "einshard comm all_reduce: size");
  const c10::cuda::CUDAGuard guard(buf.device());
  es::CommDev d = make_dev(hc, err, static_cast<int>(nblocks), 3);
  const int rc = es::comm_all_reduce(d, buf.data_ptr(), buf.numel(), es_dtype(buf), static_cast<float>(scale),
                                     static_cast<int>(nblocks), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard comm all_reduce: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

void comm_all_reduce_push(int64_t id, at::Tensor buf, double scale, int64_t nblocks, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open && buf.is_cuda() && buf.is_contiguous(), "einshard comm all_reduce (push): bad arguments");
  TORCH_CHECK(buf.scalar_type() == at::kBFloat16 || buf.scalar_type() == at::kHalf || buf.scalar_type() == at::kFloat,
              "einshard comm all_reduce (push): dtype");
  const int64_t bytes = buf.numel() * buf.element_size();
  TORCH_CHECK(bytes % 16 == 0 && es::comm_all_reduce_push_bytes(bytes / 16, hc.size) <= (long long)hc.data_bytes,
              "einshard comm all_reduce (push): size");
  const c10::cuda::CUDAGuard guard(buf.device());
  es::CommDev d = make_dev(hc, err, static_cast<int>(nblocks), 3);
  const int rc = es::comm_all_reduce_push(d, buf.data_ptr(), buf.numel(), es_dtype(buf), static_cast<float>(scale),
                                          static_cast<int>(nblocks), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard comm all_reduce (push): launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// boxes: list of (src_rank, (d0,d1,d2,d3), src_off, dst_off, (s0,s1,s2), (t0,t1,t2)) in bytes for offsets/strides
void comm_copy(int64_t id, at::Tensor src, int64_t stage_bytes, at::Tensor dst, py::list boxes, int64_t esize,
               bool reduce, bool accumulate, double scale, bool sequential, int64_t nblocks, const at::Tensor& err,
               c10::optional<at::Tensor> local) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard comm: not connected");
  TORCH_CHECK((size_t)stage_bytes <= hc.data_bytes, "einshard comm copy: staging exceeds buffer");
  TORCH_CHECK((int)py::len(boxes) <= es::kMaxBoxes, "einshard comm copy: too many boxes");
  es::CopyPlan plan;
  memset(&plan, 0, sizeof(plan));
  plan.nbox = static_cast<int>(py::len(boxes));
  plan.esize = static_cast<int>(esize);
  plan.dtype = es_dtype(dst);
  plan.accumulate = accumulate ? 1 : 0;
  plan.scale = static_cast<float>(scale);
  plan.sequential = sequential ? 1 : 0;
  for (int i = 0; i < plan.nbox; ++i) {
    py::tuple b = boxes[i].cast<py::tuple>();
    es::CopyBox& x = plan.box[i];
    x.src_rank = b[0].cast<int>();
    py::tuple dims = b[1].cast<py::tuple>();
    for (int k = 0; k < 4; ++k) x.dims[k] = dims[k].cast<int>();
    x.src_off = b[2].cast<long long>();
    x.dst_off = b[3].cast<long long>();
    py::tuple ss = b[4].cast<py::tuple>();
    py::tuple ds = b[5].cast<py::tuple>();
    for (int k = 0; k < 3; ++k) {
      x.sstr[k] = ss[k].cast<long long>();
      x.dstr[k] = ds[k].cast<long long>();
    }
    x.sstr[3] = x.dstr[3] = esize;
  }
  const c10::cuda::CUDAGuard guard(dst.device());
  const int nbar = 2 + (sequential ? plan.nbox : 0);
  es::CommDev d = make_dev(hc, err, static_cast<int>(nblocks), nbar);
  const void* sp = stage_bytes > 0 ? src.data_ptr() : nullptr;
  const int rc = reduce ? es::comm_stage_and_reduce(d, sp, stage_bytes, 0, dst.data_ptr(), plan, static_cast<int>(nblocks),
                                                    at::cuda::getCurrentCUDAStream())
                        : es::comm_stage_and_copy(d, sp, stage_bytes, 0, dst.data_ptr(), plan, static_cast<int>(nblocks),
                                                  at::cuda::getCurrentCUDAStream(),
                                                  local.has_value() ? local->data_ptr() : nullptr);
  TORCH_CHECK(rc == 0, "einshard comm copy: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// ------------------------------------------------------------------ NVLS collectives

es::NvlsDev nvls_dev(HostComm& hc, const at::Tensor& err) {
  TORCH_CHECK(hc.open && hc.mc != nullptr, "einshard NVLS: communicator has no multicast mapping");
  es::NvlsDev d;
  d.uc = static_cast<uint8_t*>(hc.local) + es::kFlagBytes;
  d.mc = static_cast<uint8_t*>(hc.mc) + es::kFlagBytes;
  d.flags = static_cast<uint32_t*>(hc.local);
  d.mcflags = static_cast<uint32_t*>(hc.mc);
  d.rank = hc.rank;
  d.size = hc.size;
  d.epoch = ++hc.nvls_epoch;
  d.nblocks = hc.nvls_blocks;
  d.err = err.data_ptr<int>();
  d.timeout_ns = g_wait_timeout_ns;
  return d;
}

// Stream-ordered wait for the completion of this heap's NVLS collectives on every rank.
void nvls_quiesce(int64_t id, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  if (hc.mc == nullptr || hc.nvls_epoch == 0) return;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(hc.device));
  es::NvlsDev d = nvls_dev(hc, err);
  d.epoch = --hc.nvls_epoch;  // the last issued collective (nvls_dev advanced the counter)
  const int rc = es::nvls_quiesce(d, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard NVLS quiesce: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

bool aligned16(const at::Tensor& t) { return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0; }

// All-reduce of a contiguous tensor through the switch: out = scale * sum over
// ranks of `in` (out may be `in`).  The heap's data region must hold the
// tensor rounded up to 16 bytes.
void nvls_all_reduce(int64_t id, const at::Tensor& in, at::Tensor out, double scale, bool two_shot,
                     const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(in.is_cuda() && in.is_contiguous() && out.is_contiguous() && out.sizes() == in.sizes() &&
                  out.scalar_type() == in.scalar_type() && aligned16(in) && aligned16(out),
              "einshard NVLS all-reduce: contiguous 16-byte aligned tensors of equal shape");
  TORCH_CHECK(in.scalar_type() == at::kBFloat16 || in.scalar_type() == at::kHalf || in.scalar_type() == at::kFloat,
              "einshard NVLS all-reduce: bf16, f16 or f32");
  const long long nbytes = in.numel() * in.element_size();
  TORCH_CHECK((size_t)((nbytes + 15) / 16 * 16) <= hc.data_bytes, "einshard NVLS all-reduce: larger than the heap");
  const c10::cuda::CUDAGuard guard(in.device());
  es::NvlsDev d = nvls_dev(hc, err);
  const int rc = es::nvls_all_reduce(d, in.data_ptr(), out.data_ptr(), nbytes, es_dtype(in), static_cast<float>(scale),
                                     two_shot ? 1 : 0, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard NVLS all-reduce: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

es::ShardLayout shard_layout(HostComm& hc, int64_t outer, int64_t inner_bytes, const std::vector<int64_t>& lens) {
  TORCH_CHECK((int)lens.size() == hc.size, "einshard NVLS: one shard length per rank");
  es::ShardLayout L;
  L.outer = outer;
  L.inner_bytes = inner_bytes;
  long long off = 0, region = 0;
  for (int q = 0; q < hc.size; ++q) {
    TORCH_CHECK(lens[q] >= 0, "einshard NVLS: negative shard length");
    L.off[q] = off;
    L.len[q] = lens[q];
    L.region[q] = region;
    off += lens[q];
    region += (outer * lens[q] * inner_bytes + 255) / 256 * 256;
  }
  L.off[hc.size] = off;
  L.total_rows = off;
  TORCH_CHECK((size_t)region <= hc.data_bytes, "einshard NVLS: shards larger than the heap");
  return L;
}

// out ([outer, sum(lens), inner], contiguous) <- every rank's `in` ([outer, lens[rank], inner]).
void nvls_all_gather(int64_t id, const at::Tensor& in, at::Tensor out, int64_t outer, int64_t inner,
                     std::vector<int64_t> lens, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(in.is_cuda() && in.is_contiguous() && out.is_contiguous() && aligned16(in) &&
                  out.scalar_type() == in.scalar_type(),
              "einshard NVLS all-gather: contiguous tensors, 16-byte aligned input");
  es::ShardLayout L = shard_layout(hc, outer, inner * in.element_size(), lens);
  TORCH_CHECK(in.numel() == outer * lens[hc.rank] * inner && out.numel() == outer * L.total_rows * inner,
              "einshard NVLS all-gather: sizes");
  const c10::cuda::CUDAGuard guard(in.device());
  es::NvlsDev d = nvls_dev(hc, err);
  const int rc = es::nvls_all_gather(d, in.data_ptr(), out.data_ptr(), L, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard NVLS all-gather: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// out ([outer, lens[rank], inner]) <- scale * sum over ranks of this rank's rows of `in` ([outer, sum(lens), inner]).
void nvls_reduce_scatter(int64_t id, const at::Tensor& in, at::Tensor out, int64_t outer, int64_t inner,
                         std::vector<int64_t> lens, double scale, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(in.is_cuda() && in.is_contiguous() && out.is_contiguous() && aligned16(out) &&
                  out.scalar_type() == in.scalar_type(),
              "einshard NVLS reduce-scatter: contiguous tensors, 16-byte aligned output");
  TORCH_CHECK(in.scalar_type() == at::kBFloat16 || in.scalar_type() == at::kHalf || in.scalar_type() == at::kFloat,
              "einshard NVLS reduce-scatter: bf16, f16 or f32");
  es::ShardLayout L = shard_layout(hc, outer, inner * in.element_size(), lens);
  TORCH_CHECK(out.numel() == outer * lens[hc.rank] * inner && in.numel() == outer * L.total_rows * inner,
              "einshard NVLS reduce-scatter: sizes");
  const c10::cuda::CUDAGuard guard(in.device());
  es::NvlsDev d = nvls_dev(hc, err);
  const int rc = es::nvls_reduce_scatter(d, in.data_ptr(), out.data_ptr(), L, es_dtype(in), static_cast<float>(scale),
                                         at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard NVLS reduce-scatter: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

void launch_gemm_nvls(HostComm& hc, const es::GemmArgs& g, int64_t reducer_clusters, int64_t lag, int64_t seg,
                      int64_t shard);

// out (every rank) = sum over the communicator's ranks of (a @ b): the wide GEMM
// and an NVLS all-reduce of its output units in one launch (gemm_nvls.cu).
void gemm_allreduce_nvls(int64_t id, const at::Tensor& a, const at::Tensor& b, at::Tensor out,
                         int64_t reducer_clusters, int64_t lag, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open && hc.mc != nullptr, "einshard fused gemm+NVLS all-reduce: no multicast mapping");
  TORCH_CHECK(a.size(0) == 1 && out.scalar_type() == at::kBFloat16 && a.scalar_type() == at::kBFloat16 &&
                  out.is_contiguous(),
              "einshard fused gemm+NVLS all-reduce: bf16, batch 1, contiguous output");
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g = gemm_args(a, b, out, 0, err);
  TORCH_CHECK(g.N % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "einshard fused gemm+NVLS all-reduce: N must be a multiple of 8");
  launch_gemm_nvls(hc, g, reducer_clusters, lag, 0, 0);
}

void launch_gemm_nvls(HostComm& hc, const es::GemmArgs& g, int64_t reducer_clusters, int64_t lag, int64_t seg,
                      int64_t shard) {
  TORCH_CHECK((size_t)g.M * g.N * 2 <= hc.data_bytes, "einshard fused gemm+NVLS: heap too small");
  TORCH_CHECK(es::gemm_nvls_units(g.M, g.N) <= es::kNvlsMaxUnits, "einshard fused gemm+NVLS: too many units");
  es::NvlsGemmJob j;
  j.heap_uc = static_cast<char*>(hc.local) + es::kFlagBytes;
  j.heap_mc = static_cast<char*>(hc.mc) + es::kFlagBytes;
  for (int p = 0; p < hc.size; ++p)
    j.ready_base[p] = reinterpret_cast<uint64_t>(static_cast<uint32_t*>(hc.bases[p]) + es::kTileReady0);
  j.reduced = static_cast<uint32_t*>(hc.local) + es::kTileReduced0;
  j.reduced_mc = static_cast<uint32_t*>(hc.mc) + es::kTileReduced0;
  j.rank = hc.rank;
  j.size = hc.size;
  j.epoch = static_cast<uint32_t>(++hc.tile_epoch);
  j.reducer_clusters = static_cast<int>(reducer_clusters);
  j.lag = static_cast<int>(lag);
  j.seg = static_cast<int>(seg);
  j.shard = static_cast<int>(shard);
  j.timeout_ns = g_wait_timeout_ns;
  const int rc = es::gemm_nvls_allreduce_launch(g, j, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard fused gemm+NVLS: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// out (this rank's rows) = reduce-scatter over the communicator's ranks of
// (a @ b) along row segments: rows [seg i + rank shard, + shard) of every
// segment i; the wide GEMM and the NVLS reduction in one launch.
void gemm_reducescatter_nvls(int64_t id, const at::Tensor& a, const at::Tensor& b, at::Tensor out, int64_t seg,
                             int64_t shard, int64_t reducer_clusters, int64_t lag, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open && hc.mc != nullptr, "einshard fused gemm+NVLS reduce-scatter: no multicast mapping");
  TORCH_CHECK(a.size(0) == 1 && a.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 &&
                  out.is_contiguous() && out.dim() == 3 && out.size(1) * hc.size == a.size(1) && out.size(2) == b.size(2),
              "einshard fused gemm+NVLS reduce-scatter: bf16, batch 1, contiguous [1, M / P, N] output");
  TORCH_CHECK(seg > 0 && shard * hc.size == seg && shard % 32 == 0 && a.size(1) % seg == 0,
              "einshard fused gemm+NVLS reduce-scatter: segments of P x (multiple of 32) rows");
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g = gemm_operand_args(a, b, 0, err);
  g.C = out.data_ptr();
  g.out_dtype = es::kDtypeBF16;
  g.ldc = out.stride(1);
  g.c_batch_stride = out.stride(0);
  const char* why = es::check_gemm_args(g);
  TORCH_CHECK(why == nullptr, "einshard fused gemm+NVLS reduce-scatter: ", why ? why : "");
  TORCH_CHECK(g.N % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "einshard fused gemm+NVLS reduce-scatter: N must be a multiple of 8");
  launch_gemm_nvls(hc, g, reducer_clusters, lag, seg, shard);
}

// out = all-reduce over the communicator's ranks of (a @ b); one fused kernel.
void gemm_allreduce(int64_t id, const at::Tensor& a, const at::Tensor& b, at::Tensor out, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard fused gemm+allreduce: communicator not connected");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && a.size(0) == 1, "einshard fused gemm+allreduce: bf16, batch 1");
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g = gemm_args(a, b, out, 0, err);
  const long long tiles = (long long)((g.M + 127) / 128) * ((g.N + 255) / 256);
  TORCH_CHECK(tiles * 128 * 256 * 2 <= (long long)hc.data_bytes && tiles <= es::kMaxTiles,
              "einshard fused gemm+allreduce: output too large for the symmetric buffer");
  const int grid = es::gemm_allreduce_grid(g);
  es::CommDev d = make_dev(hc, err, 0, 0);
  d.arrive_base = hc.arrive;
  hc.arrive += static_cast<uint32_t>(grid);
  const int rc = es::gemm_allreduce_launch(g, d, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard fused gemm+allreduce: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// out = all-reduce over the communicator's ranks of (a @ b); push-model fused
// kernel on the wide 2-SM GEMM (partials and reduced tiles travel as NVLink stores).
void gemm_allreduce_push(int64_t id, const at::Tensor& a, const at::Tensor& b, at::Tensor out, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard fused gemm+allreduce (push): communicator not connected");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && a.size(0) == 1, "einshard fused gemm+allreduce (push): bf16, batch 1");
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g = gemm_args(a, b, out, 0, err);
  TORCH_CHECK(es::gemm_push_region_bytes(g, hc.size) <= (long long)hc.data_bytes,
              "einshard fused gemm+allreduce (push): output too large for the symmetric buffer");
  const int grid = es::gemm_push_grid(g);
  es::CommDev d = make_dev(hc, err, 0, 0);
  d.arrive_base = hc.arrive;
  hc.arrive += static_cast<uint32_t>(grid);
  const int rc = es::gemm_push_allreduce_launch(g, d, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard fused gemm+allreduce (push): launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

int64_t gemm_push_region_bytes(int64_t m, int64_t n, int64_t size) {
  es::GemmArgs g;
  g.M = static_cast<int>(m);
  g.N = static_cast<int>(n);
  return es::gemm_push_region_bytes(g, static_cast<int>(size));
}

// out (this rank's rows) = reduce-scatter over the communicator's ranks of (a @ b)
// along row segments: rows [seg * i + rank * shard, ... + shard) for every i.
void gemm_reducescatter(int64_t id, const at::Tensor& a, const at::Tensor& b, at::Tensor out, int64_t seg,
                        int64_t shard, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard fused gemm+reduce-scatter: communicator not connected");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && a.size(0) == 1 && out.dim() == 3 && out.stride(2) == 1,
              "einshard fused gemm+reduce-scatter: bf16, batch 1");
  TORCH_CHECK(seg > 0 && shard * hc.size == seg && a.size(1) % seg == 0 && out.size(1) == a.size(1) / hc.size &&
                  out.size(2) == b.size(2),
              "einshard fused gemm+reduce-scatter: bad segment geometry");
  const c10::cuda::CUDAGuard guard(a.device());
  // the GEMM's full-size output view is only used for its shape; rows go to `out`
  es::GemmArgs g = gemm_operand_args(a, b, 0, err);
  g.C = out.data_ptr();
  g.out_dtype = es::kDtypeBF16;
  g.ldc = out.stride(1);
  g.c_batch_stride = out.stride(0);
  const char* why = es::check_gemm_args(g);
  TORCH_CHECK(why == nullptr, "einshard fused gemm+reduce-scatter: ", why ? why : "");
  const long long tiles = (long long)((g.M + 127) / 128) * ((g.N + 255) / 256);
  TORCH_CHECK(tiles * 128 * 256 * 2 <= (long long)hc.data_bytes && tiles <= es::kMaxTiles,
              "einshard fused gemm+reduce-scatter: output too large for the symmetric buffer");
  const int grid = es::gemm_allreduce_grid(g);
  es::CommDev d = make_dev(hc, err, 0, 0);
  d.arrive_base = hc.arrive;
  hc.arrive += static_cast<uint32_t>(grid);
  const int rc = es::gemm_allreduce_launch(g, d, at::cuda::getCurrentCUDAStream(), seg, shard);
  TORCH_CHECK(rc == 0, "einshard fused gemm+reduce-scatter: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

es::CommDev peek_dev(HostComm& hc, const at::Tensor& err);

// out = gather_rows(a_local over ranks) @ b, with the gathered rows written to
// xfull; one fused kernel (copy warps pull peers' rows while the GEMM runs).
void gemm_allgather(int64_t id, const at::Tensor& a_local, const at::Tensor& b, at::Tensor out, at::Tensor xfull,
                    int64_t seg, int64_t shard, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard fused all-gather+gemm: communicator not connected");
  TORCH_CHECK(a_local.scalar_type() == at::kBFloat16 && a_local.is_contiguous() && a_local.dim() == 3 &&
                  a_local.size(0) == 1,
              "einshard fused all-gather+gemm: contiguous bf16 [1, rows, K] shard required");
  TORCH_CHECK(xfull.is_contiguous() && xfull.scalar_type() == at::kBFloat16 && xfull.size(1) == a_local.size(1) * hc.size &&
                  xfull.size(2) == a_local.size(2),
              "einshard fused all-gather+gemm: gathered buffer shape");
  TORCH_CHECK(shard * hc.size == seg && a_local.size(1) % shard == 0, "einshard fused all-gather+gemm: segments");
  const int64_t bytes = a_local.numel() * 2;
  TORCH_CHECK((size_t)bytes <= hc.data_bytes, "einshard fused all-gather+gemm: shard larger than the symmetric region");
  const c10::cuda::CUDAGuard guard(a_local.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  // peers finished reading this rank's region (previous op), then stage the shard
  es::CommDev prev = peek_dev(hc, err);
  int rc = es::comm_wait_peers(prev, es::kFlagDone, hc.epoch, stream);
  TORCH_CHECK(rc == 0, "einshard fused all-gather+gemm: wait launch failed (", rc, ")");
  void* region = static_cast<char*>(hc.local) + es::kFlagBytes;
  TORCH_CHECK(cudaMemcpyAsync(region, a_local.data_ptr(), bytes, cudaMemcpyDeviceToDevice, stream) == cudaSuccess,
              "einshard fused all-gather+gemm: staging copy failed");
  es::GemmArgs g = gemm_args(xfull, b, out, 0, err);
  TORCH_CHECK(g.out_dtype == es::kDtypeBF16, "einshard fused all-gather+gemm: bf16 output");
  const int grid = es::gemm_allgather_grid(g);
  es::CommDev d = make_dev(hc, err, 0, 0);
  d.arrive_base = hc.arrive;
  hc.arrive += static_cast<uint32_t>(grid);
  rc = es::gemm_allgather_launch(g, d, xfull.data_ptr(), static_cast<int>(a_local.size(1) / shard), shard, stream);
  TORCH_CHECK(rc == 0, "einshard fused all-gather+gemm: launch failed (", rc, ")");
  g_launches.fetch_add(2, std::memory_order_relaxed);
}


// ------------------------------------------------------------------ FFT

const float2* f2(const at::Tensor& t) { return reinterpret_cast<const float2*>(t.data_ptr()); }
float2* f2m(at::Tensor& t) { return reinterpret_cast<float2*>(t.data_ptr()); }

void check_twiddles(const at::Tensor& tw, int64_t n, const at::Tensor& like) {
  TORCH_CHECK(tw.is_cuda() && tw.scalar_type() == at::kComplexFloat && tw.is_contiguous() && tw.numel() == n &&
                  tw.get_device() == like.get_device(),
              "einshard fft: twiddle table must be a contiguous complex64 CUDA tensor of length n");
}

// out = scale * DFT_dim(in) (unnormalised inverse when `inverse`); in and out
// are contiguous complex64 tensors of the same shape (out may alias in).
void fft_c2c(const at::Tensor& in, at::Tensor out, int64_t dim, bool inverse, const at::Tensor& tw, double scale) {
  TORCH_CHECK(in.is_cuda() && in.scalar_type() == at::kComplexFloat && in.is_contiguous(),
              "einshard fft: contiguous complex64 CUDA input required");
  TORCH_CHECK(out.sizes() == in.sizes() && out.scalar_type() == at::kComplexFloat && out.is_contiguous() &&
                  out.get_device() == in.get_device(),
              "einshard fft: output must match the input");
  TORCH_CHECK(dim >= 0 && dim < in.dim(), "einshard fft: bad dim");
  const int64_t n = in.size(dim);
  TORCH_CHECK(es::fft_supported(n), "einshard fft: length ", n, " is not a supported power of two");
  check_twiddles(tw, n, in);
  long long outer = 1, inner = 1;
  for (int64_t d = 0; d < dim; ++d) outer *= in.size(d);
  for (int64_t d = dim + 1; d < in.dim(); ++d) inner *= in.size(d);
  if (outer * inner == 0) return;
  const c10::cuda::CUDAGuard guard(in.device());
  es::FftLines f;
  f.in = f2(in);
  f.out = f2m(out);
  f.n = n;
  f.outer = outer;
  f.inner = inner;
  f.in_os = f.out_os = n * inner;
  f.in_ps = f.out_ps = inner;
  f.in_is = f.out_is = 1;
  f.tw = f2(tw);
  f.scale = static_cast<float>(scale);
  f.inverse = inverse ? 1 : 0;
  const int rc = es::fft_lines(f, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard fft: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

es::CommDev peek_dev(HostComm& hc, const at::Tensor& err) {
  es::CommDev d;
  d.rank = hc.rank;
  d.size = hc.size;
  for (int p = 0; p < es::kMaxRanks; ++p) {
    d.flags[p] = p < hc.size ? reinterpret_cast<uint64_t>(hc.bases[p]) : 0;
    d.data[p] = p < hc.size ? reinterpret_cast<uint64_t>(hc.bases[p]) + es::kFlagBytes : 0;
  }
  d.epoch = hc.epoch;
  d.bar_base = hc.bar;
  d.arrive_base = hc.arrive;
  d.err = err.data_ptr<int>();
  d.timeout_ns = g_wait_timeout_ns;
  return d;
}

// The first `nbytes` of this rank's symmetric data region as a uint8 tensor.
// Writes into it must follow comm_acquire (peers may still read the previous op).
at::Tensor comm_region(int64_t id, int64_t nbytes) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open && nbytes >= 0 && (size_t)nbytes <= hc.data_bytes, "einshard comm region: size");
  void* p = static_cast<char*>(hc.local) + es::kFlagBytes;
  return torch::from_blob(p, {nbytes}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, hc.device));
}

// Stream-ordered wait until every peer finished reading this rank's region for
// the last op on the communicator.
void comm_acquire(int64_t id, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard comm: not connected");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(hc.device));
  es::CommDev d = peek_dev(hc, err);
  const int rc = es::comm_wait_peers(d, es::kFlagDone, hc.epoch, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard comm acquire: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// Slab transpose fused with the FFT along the exchanged axis (fft.h FftSlab).
void fft_slab(int64_t id, at::Tensor out, int64_t n, int64_t A, int64_t B, int64_t C, int64_t D, int64_t Dl,
              int64_t doff, int64_t mode, const at::Tensor& tw, double scale, bool inverse, const at::Tensor& err) {
  HostComm& hc = comm_ref(id);
  TORCH_CHECK(hc.open, "einshard fft slab: communicator not connected");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kComplexFloat && out.is_contiguous(),
              "einshard fft slab: contiguous complex64 output required");
  TORCH_CHECK(es::fft_supported(n) && n % hc.size == 0 && D % hc.size == 0 && Dl * hc.size == D,
              "einshard fft slab: unsupported sizes");
  TORCH_CHECK(out.numel() == A * B * C * Dl * n, "einshard fft slab: output size");
  TORCH_CHECK((size_t)(A * B * C * D * (n / hc.size)) * 8 <= hc.data_bytes, "einshard fft slab: region too small");
  check_twiddles(tw, n, out);
  const c10::cuda::CUDAGuard guard(out.device());
  es::FftSlab f;
  f.out = f2m(out);
  f.n = n;
  f.A = A;
  f.B = B;
  f.C = C;
  f.D = D;
  f.Dl = Dl;
  f.doff = doff;
  f.mode = static_cast<int>(mode);
  f.tw = f2(tw);
  f.scale = static_cast<float>(scale);
  f.inverse = inverse ? 1 : 0;
  es::CommDev d = make_dev(hc, err, 0, 0);
  const long long lines = A * B * C * Dl;
  d.arrive_base = hc.arrive;
  hc.arrive += static_cast<uint32_t>(es::fft_grid(n, lines));
  const int rc = es::fft_slab(d, f, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard fft slab: launch failed (", rc, ")");
  g_launches.fetch_add(2, std::memory_order_relaxed);
}

// ------------------------------------------------------------------ convolution

// out[B, Hout, Wout, O] = conv2d(x[B, Hin, Win, C], w[O, KH, KW, C]) + bias, zero padding (ph, pw).
// out = conv(x, w) + bias with zero padding (ph, ph_hi) rows and (pw, pw_hi)
// columns (hi < 0: the same as lo); kernel 0 picks the CTA-pair kernel with
// resident weights where it fits, 1 forces conv.cu's kernel.
// ghosts: empty, or [B][gtop + gbot][W][C] rows that continue x above and below
// (the CTA-pair kernel reads them in place of a haloed copy of x).
// ghost_wpitch / ghost_w0: ghost rows wider than x, x's columns from ghost_w0;
// out_w0: the computed columns go to columns out_w0 .. of out (whose width
// may exceed the conv's; 0 with out as wide as the conv: the whole output).
void conv2d_implicit(const at::Tensor& x, const at::Tensor& w, const at::Tensor& bias, at::Tensor out, int64_t ph,
                     int64_t pw, int64_t ph_hi, int64_t pw_hi, int64_t kernel, const at::Tensor& ghosts, int64_t gtop,
                     int64_t gbot, int64_t ghost_w0, int64_t out_w0, const at::Tensor& err) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda() && x.dim() == 4 && w.dim() == 4 && out.dim() == 4,
              "einshard conv: 4-D CUDA tensors required");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && out.is_contiguous(), "einshard conv: contiguous NHWC required");
  TORCH_CHECK(x.scalar_type() == w.scalar_type() && x.scalar_type() == out.scalar_type() &&
                  (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf),
              "einshard conv: bf16/fp16 tensors of one dtype required");
  TORCH_CHECK(w.size(3) == x.size(3), "einshard conv: channel mismatch");
  es::ConvArgs a;
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.out = out.data_ptr();
  a.dtype = dtype_code(x.scalar_type());
  a.B = x.size(0);
  a.Hin = x.size(1);
  a.Win = x.size(2);
  a.C = x.size(3);
  a.O = w.size(0);
  a.KH = w.size(1);
  a.KW = w.size(2);
  a.ph = static_cast<int>(ph);
  a.pw = static_cast<int>(pw);
  if (bias.numel() > 0) {
    TORCH_CHECK(bias.is_cuda() && bias.scalar_type() == at::kFloat && bias.is_contiguous() && bias.numel() == a.O,
                "einshard conv: bias must be a contiguous float32 CUDA tensor of length O");
    a.bias = bias.data_ptr<float>();
  }
  a.err = err.data_ptr<int>();
  a.num_sms = num_sms(x.get_device());
  a.persistent = g_small_persistent;
  a.ph_hi = static_cast<int>(ph_hi);
  a.pw_hi = static_cast<int>(pw_hi);
  a.kernel = static_cast<int>(kernel);
  a.prof = g_prof;
  if (gtop + gbot > 0) {
    TORCH_CHECK(ghosts.is_cuda() && ghosts.is_contiguous() && ghosts.dim() == 4 && ghosts.scalar_type() == x.scalar_type() &&
                    ghosts.size(0) == x.size(0) && ghosts.size(1) == gtop + gbot && ghosts.size(2) >= x.size(2) &&
                    ghosts.size(3) == x.size(3) && gtop >= 0 && gbot >= 0,
                "einshard conv: ghosts must be a contiguous [B, gtop + gbot, W, C] tensor like x");
    a.ghosts = ghosts.data_ptr();
    a.gtop = static_cast<int>(gtop);
    a.gbot = static_cast<int>(gbot);
  }
  if (gtop + gbot > 0) {
    TORCH_CHECK(ghost_w0 >= 0 && ghost_w0 + x.size(2) <= ghosts.size(2), "einshard conv: ghost column range");
    a.ghost_wpitch = static_cast<int>(ghosts.size(2));
    a.ghost_w0 = static_cast<int>(ghost_w0);
  }
  const char* why = es::check_conv_args(a);
  TORCH_CHECK(why == nullptr, "einshard conv: ", why ? why : "");
  const int Hout = es::conv_hout(a);
  const int Wout = es::conv_wout(a);
  if (out.size(2) != Wout || out_w0 != 0) {  // the conv fills columns out_w0 .. out_w0 + Wout of out
    TORCH_CHECK(out_w0 >= 0 && out_w0 + Wout <= out.size(2), "einshard conv: output column range");
    a.out_wpitch = static_cast<int>(out.size(2));
    a.out_w0 = static_cast<int>(out_w0);
  }
  TORCH_CHECK(out.size(0) == a.B && out.size(1) == Hout && out.size(2) >= Wout && out.size(3) == a.O,
              "einshard conv: output shape");
  const c10::cuda::CUDAGuard guard(x.device());
  const int rc = es::conv_launch(a, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard conv: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

void wait_probe(const at::Tensor& flag, int64_t target, int64_t timeout_ns, at::Tensor result, const at::Tensor& err) {
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && result.is_cuda() && result.scalar_type() == at::kInt,
              "einshard wait_probe: int32 CUDA tensors required");
  const c10::cuda::CUDAGuard guard(flag.device());
  const int rc = es::wait_probe(flag.data_ptr<int>(), static_cast<int>(target), err.data_ptr<int>(), timeout_ns,
                                result.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard wait_probe: launch failed (", rc, ")");
}

// The same bounded wait, recording its code in the status word of the
// allocation-free GEMM entry point (tests of es_gemm_bf16_noalloc_status).
void wait_probe_noalloc_status(const at::Tensor& flag, int64_t target, int64_t timeout_ns, at::Tensor result) {
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt && result.is_cuda() && result.scalar_type() == at::kInt,
              "einshard wait_probe_noalloc_status: int32 CUDA tensors required");
  const c10::cuda::CUDAGuard guard(flag.device());
  int* status = es::noalloc_status_word();
  TORCH_CHECK(status != nullptr, "einshard wait_probe_noalloc_status: no scratch address");
  const int rc = es::wait_probe(flag.data_ptr<int>(), static_cast<int>(target), status, timeout_ns,
                                result.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard wait_probe_noalloc_status: launch failed (", rc, ")");
}

// out = x (contiguous) rolled by shifts[d] along every dim d, one kernel.
void roll_copy(const at::Tensor& x, at::Tensor out, std::vector<int64_t> shifts) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && out.is_contiguous() && out.sizes() == x.sizes() &&
                  out.scalar_type() == x.scalar_type() && (int64_t)shifts.size() == x.dim() &&
                  x.dim() >= 1 && x.dim() <= es::kCopyMaxRank + 1,
              "einshard roll: contiguous tensors of equal shape, one shift per dim");
  const c10::cuda::CUDAGuard guard(x.device());
  std::vector<long long> size(x.sizes().begin(), x.sizes().end()), shift(shifts.begin(), shifts.end());
  const int rc = es::roll_copy(x.data_ptr(), out.data_ptr(), static_cast<int>(x.element_size()),
                               static_cast<int>(x.dim()), size.data(), shift.data(), num_sms(x.get_device()),
                               at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard roll: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// out (contiguous) = view (any strides, rank <= 8), one gather kernel.
void strided_copy(const at::Tensor& view, at::Tensor out) {
  TORCH_CHECK(view.is_cuda() && out.is_cuda() && out.is_contiguous() && out.sizes() == view.sizes() &&
                  out.scalar_type() == view.scalar_type() && view.dim() <= es::kCopyMaxRank,
              "einshard strided_copy: bad arguments");
  if (view.numel() == 0) return;
  long long size[es::kCopyMaxRank], stride[es::kCopyMaxRank];
  for (int64_t d = 0; d < view.dim(); ++d) {
    size[d] = view.size(d);
    stride[d] = view.stride(d);
  }
  const int rank = view.dim() == 0 ? 1 : static_cast<int>(view.dim());
  if (view.dim() == 0) {
    size[0] = 1;
    stride[0] = 1;
  }
  const c10::cuda::CUDAGuard guard(view.device());
  const int rc = es::strided_gather(view.data_ptr(), out.data_ptr(), static_cast<int>(view.element_size()), rank, size,
                                    stride, num_sms(view.get_device()), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard strided_copy: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

int64_t comm_data_bytes(int64_t id) { return static_cast<int64_t>(comm_ref(id).data_bytes); }

}  // namespace

// dw (fp32 [O][KH][KW][C], zeroed here) = weight gradient of the implicit-GEMM
// conv with input x [B][Hin][Win][C], output gradient dy [B][Hout][Wout][O].
void conv2d_wgrad(const at::Tensor& x, const at::Tensor& dy, at::Tensor dw, int64_t ph, int64_t pw, int64_t ph_hi,
                  int64_t pw_hi, const at::Tensor& err) {
  TORCH_CHECK(x.is_cuda() && dy.is_cuda() && dw.is_cuda() && x.dim() == 4 && dy.dim() == 4 && dw.dim() == 4,
              "einshard conv wgrad: 4-D CUDA tensors required");
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous() && dw.is_contiguous(), "einshard conv wgrad: contiguous required");
  TORCH_CHECK(x.scalar_type() == dy.scalar_type() && (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf),
              "einshard conv wgrad: bf16/fp16 x and dy of one dtype required");
  TORCH_CHECK(dw.scalar_type() == at::kFloat, "einshard conv wgrad: fp32 dw required");
  es::ConvWgradArgs a;
  a.x = x.data_ptr();
  a.dy = dy.data_ptr();
  a.dw = dw.data_ptr<float>();
  a.dtype = dtype_code(x.scalar_type());
  a.B = x.size(0);
  a.Hin = x.size(1);
  a.Win = x.size(2);
  a.C = x.size(3);
  a.O = dw.size(0);
  a.KH = dw.size(1);
  a.KW = dw.size(2);
  a.ph = static_cast<int>(ph);
  a.pw = static_cast<int>(pw);
  a.ph_hi = static_cast<int>(ph_hi);
  a.pw_hi = static_cast<int>(pw_hi);
  a.err = err.data_ptr<int>();
  a.num_sms = num_sms(x.get_device());
  TORCH_CHECK(dw.size(3) == a.C, "einshard conv wgrad: channel mismatch");
  const char* why = es::check_conv_wgrad_args(a);
  TORCH_CHECK(why == nullptr, "einshard conv wgrad: ", why ? why : "");
  const int Hout = es::conv_hout(a);
  const int Wout = es::conv_wout(a);
  TORCH_CHECK(dy.size(0) == a.B && dy.size(1) == Hout && dy.size(2) == Wout && dy.size(3) == a.O,
              "einshard conv wgrad: output-gradient shape");
  const c10::cuda::CUDAGuard guard(x.device());
  dw.zero_();
  const int rc = es::conv_wgrad_launch(a, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard conv wgrad: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "einshard sm_100a native kernels";
  m.def("gemm", &gemm, "C = act(A @ B), tcgen05 GEMM (A [B,M,K], B [B,K,N])");
  m.def("gemm_out", &gemm_out, "gemm into a preallocated row-major output");
  m.def("symm_multicast_supported", &symm_multicast_supported, "whether a device supports NVLS multicast objects");
  m.def("symm_prepare", &symm_prepare, "communicator over a symmetric heap, phase 1: returns (id, error)");
  m.def("symm_exchange", &symm_exchange, "phase 2: exchange descriptors, map peers, join the multicast team");
  m.def("symm_bind", &symm_bind, "phase 3: bind this rank's memory to the multicast object");
  m.def("symm_finish", &symm_finish, "phase 4: map the multicast object, zero the flags");
  m.def("comm_destroy", &comm_destroy, "unmap and free");
  m.def("comm_has_multicast", &comm_has_multicast, "whether the communicator has an NVLS multicast mapping");
  m.def("gemm_reducescatter_nvls", &gemm_reducescatter_nvls,
        "wide GEMM whose output row segments are reduce-scattered through the NVSwitch in the same launch");
  m.def("gemm_allreduce_nvls", &gemm_allreduce_nvls,
        "wide GEMM whose output units are all-reduced through the NVSwitch in the same launch");
  m.def("nvls_quiesce", &nvls_quiesce, "wait until every rank completed this heap's NVLS collectives");
  m.def("nvls_all_reduce", &nvls_all_reduce, "all-reduce through the NVSwitch (multimem), one- or two-shot");
  m.def("nvls_all_gather", &nvls_all_gather, "all-gather along a dimension through multicast stores");
  m.def("nvls_reduce_scatter", &nvls_reduce_scatter, "reduce-scatter along a dimension through the NVSwitch");
  m.def("comm_all_reduce", &comm_all_reduce, "two-shot NVLink all-reduce in place");
  m.def("comm_all_reduce_push", &comm_all_reduce_push, "two-shot NVLink all-reduce in place, stores only");
  m.def("comm_copy", &comm_copy, "stage + pull strided boxes from peers (copy, accumulate or reduce)",
        py::arg("id"), py::arg("src"), py::arg("stage_bytes"), py::arg("dst"), py::arg("boxes"), py::arg("esize"),
        py::arg("reduce"), py::arg("accumulate"), py::arg("scale"), py::arg("sequential"), py::arg("nblocks"),
        py::arg("err"), py::arg("local") = py::none());
  m.def("gemm_allreduce", &gemm_allreduce, "fused tcgen05 GEMM + NVLink all-reduce (bf16)");
  m.def("conv2d_wgrad", &conv2d_wgrad, "weight gradient of the implicit-GEMM conv (split-K tcgen05, fp32 out)");
  m.def("conv2d_implicit", &conv2d_implicit, "implicit-GEMM NHWC conv2d on tcgen05 (stride 1)");
  m.def("conv_pair_otile", [](int64_t C, int64_t O, int64_t KH, int64_t KW) {
        return es::conv_pair_otile(static_cast<int>(C), static_cast<int>(O), static_cast<int>(KH), static_cast<int>(KW));
      }, "output-channel tile of the CTA-pair conv for this shape (0: the kernel does not take it)");
  m.def("roll_copy", &roll_copy, "cyclic roll along several dims in one kernel");
  m.def("gemm_silu", &gemm_silu, "(silu(a @ b), a @ b), fused on the wide kernel when it runs the GEMM");
  m.def("silu_forward", &silu_forward, "elementwise silu");
  m.def("silu_backward", &silu_backward, "grad * silu'(h)");
  m.def("wait_probe", &wait_probe, "bounded wait on a flag (tests the timeout path)");
  m.def("wait_probe_noalloc_status", &wait_probe_noalloc_status,
        "bounded wait recording into the allocation-free GEMM's status word (tests)");
  m.def("strided_copy", &strided_copy, "materialise a strided view contiguously");
  m.def("fft_c2c", &fft_c2c, "complex64 FFT along one dim (powers of two up to 1024)");
  m.def("comm_region", &comm_region, "this rank's symmetric data region as a uint8 tensor");
  m.def("comm_acquire", &comm_acquire, "wait until peers finished reading this rank's region");
  m.def("fft_slab", &fft_slab, "slab transpose fused with the FFT along the exchanged axis");
  m.def("gemm_reducescatter", &gemm_reducescatter, "fused tcgen05 GEMM + NVLink reduce-scatter of row segments (bf16)");
  m.def("gemm_allgather", &gemm_allgather, "fused all-gather of row shards + tcgen05 GEMM (bf16)");
  m.def("gemm_allreduce_push", &gemm_allreduce_push, "push-model fused wide GEMM + NVLink all-reduce (bf16)");
  m.def("gemm_push_region_bytes", &gemm_push_region_bytes, "symmetric bytes the push all-reduce needs");
  m.def("comm_data_bytes", &comm_data_bytes, "data capacity of a communicator");
  m.def("set_gemm_pair_mode", [](int64_t m) { g_pair_mode = static_cast<int>(m); },
        "-1 heuristic, 0 force 1-SM, 1 force 2-SM GEMM kernel");
  m.def("set_gemm_group_m", [](int64_t v) { g_group_m = static_cast<int>(v); }, "raster group height (0 default)");
  m.def("set_gemm_split", [](int64_t v) { g_split = static_cast<int>(v); }, "wide-kernel cluster split (0/1/2)");
  m.def("set_gemm_profile", [](const at::Tensor& t) {
        g_prof = t.numel() >= 8 ? reinterpret_cast<unsigned long long*>(t.data_ptr()) : nullptr;
      }, "int64 CUDA tensor of >= 8 wait-cycle counters for the wide GEMM and the pair conv (empty tensor: off)");
  m.def("set_gemm_persistent", [](int64_t v) { g_persistent = static_cast<int>(v); }, "wide kernel: 1 persistent, 0 one tile per cluster, -1 by K");
  m.def("set_small_persistent", [](int64_t v) { g_small_persistent = static_cast<int>(v); },
        "1-SM GEMM and conv: 1 persistent CTAs, 0 one tile per CTA");
  m.def("set_wait_timeout_ns", [](int64_t v) { g_wait_timeout_ns = static_cast<uint64_t>(v > 0 ? v : 1); },
        "bound (ns) of every device-side wait on a peer rank");
  m.def("get_wait_timeout_ns", []() { return static_cast<int64_t>(g_wait_timeout_ns); });
  m.def("set_gemm_streamk", [](int64_t v) { g_streamk = static_cast<int>(v); },
        "stream-K wide GEMM: -1 split the partial last wave (default), 1 split every tile, 0 never");
  m.def("gemm_plan",
        [](int64_t M, int64_t N, int64_t K, int64_t batch, bool a_mn, bool b_mn, int64_t num_sms) {
          es::GemmArgs g;
          g.M = static_cast<int>(M);
          g.N = static_cast<int>(N);
          g.K = static_cast<int>(K);
          g.batch = static_cast<int>(batch);
          g.a_mn = a_mn ? 1 : 0;
          g.b_mn = b_mn ? 1 : 0;
          g.num_sms = static_cast<int>(num_sms);
          g.pair = g_pair_mode;
          g.persistent = g_persistent;
          const es::GemmPlanInfo info = es::gemm_plan_info(g, g_streamk);
          py::dict d;
          d["kernel"] = info.kernel;
          d["swapped"] = info.swapped;
          d["persistent"] = info.persistent;
          d["sk_first"] = info.sk_first;
          d["sk_iters"] = info.sk_iters;
          d["tail_tiles"] = info.tail_tiles;
          d["clusters"] = info.clusters;
          return d;
        },
        "kernel choice for a GEMM shape (no launch; runs without a GPU)");
  m.def("fft_slab_sources",
        [](int64_t mode, int64_t n, int64_t A, int64_t B, int64_t C, int64_t D, int64_t Dl, int64_t doff,
           int64_t size) {
          es::FftSlab f{};
          f.mode = static_cast<int>(mode);
          f.n = n;
          f.A = A;
          f.B = B;
          f.C = C;
          f.D = D;
          f.Dl = Dl;
          f.doff = doff;
          const int64_t total = A * B * C * Dl * n;
          at::Tensor out_off = at::empty({total}, at::kLong), src_off = at::empty({total}, at::kLong);
          at::Tensor src_rank = at::empty({total}, at::kInt);
          const int rc = es::fft_slab_sources(f, static_cast<int>(size),
                                              reinterpret_cast<long long*>(out_off.data_ptr<int64_t>()),
                                              src_rank.data_ptr<int>(),
                                              reinterpret_cast<long long*>(src_off.data_ptr<int64_t>()));
          TORCH_CHECK(rc == 0, "fft_slab_sources: unsupported geometry");
          return py::make_tuple(out_off, src_rank, src_off);
        },
        "host walk of the slab exchange's loads: output offsets, source ranks and offsets");
  m.def("gemm_allgather_row_order",
        [](int64_t rank, int64_t size, int64_t segments, int64_t shard) {
          return es::gemm_allgather_row_order(static_cast<int>(rank), static_cast<int>(size),
                                              static_cast<int>(segments), shard);
        },
        "row-block order of the fused all-gather GEMM on one rank (host walk)");
  m.def("gemm_wide_schedule",
        [](int64_t M, int64_t N, int64_t K, int64_t num_sms) {
          es::GemmArgs g;
          g.M = static_cast<int>(M);
          g.N = static_cast<int>(N);
          g.K = static_cast<int>(K);
          g.num_sms = static_cast<int>(num_sms);
          g.pair = g_pair_mode;
          g.persistent = g_persistent;
          g.group_m = g_group_m;
          py::list out;
          for (const es::GemmSegment& sg : es::gemm_wide_schedule(g, g_streamk))
            out.append(py::make_tuple(sg.launch, sg.cluster, sg.pair_tile, sg.m0, sg.n0, sg.kb0, sg.kb1));
          return out;
        },
        "wide-kernel schedule (launch, cluster, pair tile, m0, n0, kb0, kb1) of a GEMM shape (host walk)");
  m.def("set_gemm_sleep_ns", [](int64_t v) { g_sleep_ns = static_cast<int>(v); }, "wide-kernel epilogue back-off ns");
  m.def("set_tma_l2_promotion", [](int64_t v) { es::tma_l2_promotion() = static_cast<int>(v); },
        "L2 promotion of TMA loads: 0 none, 1 64B, 2 128B, 3 256B (tuning)");
  m.def("launch_count", []() { return g_launches.load(); }, "native kernel launches so far");
}
