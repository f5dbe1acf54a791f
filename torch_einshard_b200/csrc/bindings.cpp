// Torch bindings of the native einshard kernels (module torch_einshard_b200._C).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>

#include "gemm.h"

namespace {

// Number of native kernel launches issued through these bindings (all devices).
std::atomic<long long> g_launches{0};

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

void run_gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, int64_t act, const at::Tensor& err) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "einshard native gemm: CUDA tensors required");
  TORCH_CHECK(a.dim() == 3 && b.dim() == 3 && out.dim() == 3, "einshard native gemm: 3-D operands required");
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "einshard native gemm: operand dtypes differ");
  TORCH_CHECK(a.size(0) == b.size(0) && a.size(2) == b.size(1), "einshard native gemm: shape mismatch");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == a.size(1) && out.size(2) == b.size(2),
              "einshard native gemm: output shape mismatch");
  TORCH_CHECK(out.stride(2) == 1, "einshard native gemm: output must be row-major");
  const c10::cuda::CUDAGuard guard(a.device());
  es::GemmArgs g;
  g.A = a.data_ptr();
  g.B = b.data_ptr();
  g.C = out.data_ptr();
  g.dtype = dtype_code(a.scalar_type());
  TORCH_CHECK(g.dtype != es::kDtypeF32, "einshard native gemm: bf16/fp16 operands required");
  g.out_dtype = dtype_code(out.scalar_type());
  g.batch = a.size(0);
  g.M = a.size(1);
  g.K = a.size(2);
  g.N = b.size(2);
  operand_layout(a, true, g.a_mn, g.lda, g.a_batch_stride);
  operand_layout(b, false, g.b_mn, g.ldb, g.b_batch_stride);
  g.ldc = out.stride(1);
  g.c_batch_stride = out.stride(0);
  g.act = static_cast<int>(act);
  g.err = err.data_ptr<int>();
  g.num_sms = num_sms(a.get_device());
  const char* why = es::check_gemm_args(g);
  TORCH_CHECK(why == nullptr, "einshard native gemm: ", why ? why : "");
  const int rc = es::gemm_launch(g, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "einshard native gemm: launch failed (", rc, ")");
  g_launches.fetch_add(1, std::memory_order_relaxed);
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

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "einshard sm_100a native kernels";
  m.def("gemm", &gemm, "C = act(A @ B), tcgen05 GEMM (A [B,M,K], B [B,K,N])");
  m.def("gemm_out", &gemm_out, "gemm into a preallocated row-major output");
  m.def("launch_count", []() { return g_launches.load(); }, "native kernel launches so far");
}
