// Python bindings of the sm_100a kernel library.  Tensors are checked and translated into raw
// pointers/strides here; the CUDA translation units never include torch headers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common/host.h"
#include "gemm/api.h"

namespace {

using torch::Tensor;

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
}

// A operand of a GEMM given as the math matrix a[M, K].
ttb::Operand a_operand(const Tensor& a) {
  check_bf16(a, "A");
  TORCH_CHECK(a.dim() == 2, "A must be 2-D");
  if (a.stride(1) == 1 && (a.size(0) == 1 || a.stride(0) >= a.size(1)))
    return {a.data_ptr(), a.stride(0), false};
  TORCH_CHECK(a.stride(0) == 1, "A must have a unit stride in one dimension");
  return {a.data_ptr(), a.stride(1), true};
}
// B operand given as the math matrix b[K, N] (result = a @ b).
ttb::Operand b_operand(const Tensor& b) {
  check_bf16(b, "B");
  TORCH_CHECK(b.dim() == 2, "B must be 2-D");
  if (b.stride(0) == 1 && (b.size(1) == 1 || b.stride(1) >= b.size(0)))
    return {b.data_ptr(), b.stride(1), false};  // stored [N][K]
  TORCH_CHECK(b.stride(1) == 1, "B must have a unit stride in one dimension");
  return {b.data_ptr(), b.stride(0), true};  // stored [K][N]
}

// out = alpha * (a @ b + bias) + beta * c     (out/c: bf16 or fp32, row-major rows)
void mm(const Tensor& a, const Tensor& b, Tensor& out, const c10::optional<Tensor>& c, double alpha, double beta,
        const c10::optional<Tensor>& bias) {
  const c10::cuda::CUDAGuard guard(a.device());
  const auto A = a_operand(a);
  const auto B = b_operand(b);
  const int M = a.size(0), K = a.size(1), N = b.size(1);
  TORCH_CHECK(b.size(0) == K, "inner dimensions differ");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "bad output");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32, "out dtype");
  const void* cp = nullptr;
  long long ldc = 0;
  bool c_f32 = false;
  if (c.has_value() && beta != 0.0) {
    const Tensor& ct = *c;
    TORCH_CHECK(ct.dim() == 2 && ct.size(0) == M && ct.size(1) == N && ct.stride(1) == 1, "bad C");
    TORCH_CHECK(ct.scalar_type() == torch::kBFloat16 || ct.scalar_type() == torch::kFloat32, "C dtype");
    cp = ct.data_ptr();
    ldc = ct.stride(0);
    c_f32 = ct.scalar_type() == torch::kFloat32;
  }
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->is_contiguous() && bias->numel() == N, "bias");
    bp = bias->data_ptr<float>();
  }
  ttb::gemm_linear(A, B, M, N, K, out.data_ptr(), out.stride(0), out.scalar_type() == torch::kFloat32, cp, ldc,
                   c_f32, static_cast<float>(alpha), static_cast<float>(beta), bp, cur_stream());
}

// h = l*r (mode 0) / silu(l)*r (mode 1) with l = x wl^T (+bl), r = x wr^T (+br)
void bilinear(const Tensor& x, const Tensor& wl, const Tensor& wr, const c10::optional<Tensor>& bl,
              const c10::optional<Tensor>& br, int64_t mode, Tensor& h, const c10::optional<Tensor>& lo,
              const c10::optional<Tensor>& ro) {
  const c10::cuda::CUDAGuard guard(x.device());
  const auto X = a_operand(x);
  const auto WL = b_operand(wl.t());
  const auto WR = b_operand(wr.t());
  const int M = x.size(0), K = x.size(1), N = wl.size(0);
  TORCH_CHECK(wl.size(1) == K && wr.size(0) == N && wr.size(1) == K, "weight shapes");
  check_bf16(h, "h");
  TORCH_CHECK(h.is_contiguous() && h.size(0) == M && h.size(1) == N, "h shape");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0, "h must be 16-byte aligned");
  void* lp = nullptr;
  void* rp = nullptr;
  if (lo.has_value()) {
    TORCH_CHECK(lo->is_contiguous() && lo->sizes() == h.sizes() && lo->scalar_type() == torch::kBFloat16, "lo");
    lp = lo->data_ptr();
  }
  if (ro.has_value()) {
    TORCH_CHECK(ro->is_contiguous() && ro->sizes() == h.sizes() && ro->scalar_type() == torch::kBFloat16, "ro");
    rp = ro->data_ptr();
  }
  const float* blp = bl.has_value() ? bl->data_ptr<float>() : nullptr;
  const float* brp = br.has_value() ? br->data_ptr<float>() : nullptr;
  TORCH_CHECK((blp == nullptr) == (brp == nullptr), "both biases or neither");
  ttb::gemm_bilinear(X, WL, WR, M, N, K, h.data_ptr(), lp, rp, h.stride(0), blp, brp, static_cast<int>(mode),
                     cur_stream());
}

// dl, dr from dH = dy @ wd (wd: [d_out, N] weight of the down projection)
void bilinear_grad(const Tensor& dy, const Tensor& wd, const Tensor& l, const Tensor& r, Tensor& dl, Tensor& dr,
                   int64_t mode) {
  const c10::cuda::CUDAGuard guard(dy.device());
  const auto DY = a_operand(dy);
  const auto WD = b_operand(wd);
  const int M = dy.size(0), K = dy.size(1), N = wd.size(1);
  TORCH_CHECK(wd.size(0) == K, "wd shape");
  for (const Tensor* t : std::initializer_list<const Tensor*>{&l, &r, &dl, &dr}) {
    check_bf16(*t, "bilinear factor");
    TORCH_CHECK(t->is_contiguous() && t->size(0) == M && t->size(1) == N, "factor shape");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "bilinear factors must be 16-byte aligned");
  }
  ttb::gemm_bilinear_grad(DY, WD, M, N, K, l.data_ptr(), r.data_ptr(), dl.data_ptr(), dr.data_ptr(), l.stride(0),
                          static_cast<int>(mode), cur_stream());
}

int64_t status() { return static_cast<int64_t>(ttb::status_read_and_reset()); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tensor_train_ing_b200 sm_100a kernels (tcgen05 / TMEM / TMA)";
  m.def("mm", &mm, "out = alpha*(a@b + bias) + beta*c on the tcgen05 GEMM", py::arg("a"), py::arg("b"),
        py::arg("out"), py::arg("c") = py::none(), py::arg("alpha") = 1.0, py::arg("beta") = 0.0,
        py::arg("bias") = py::none());
  m.def("bilinear", &bilinear, "dual-B GEMM forming the bilinear hidden layer");
  m.def("bilinear_grad", &bilinear_grad, "dH GEMM fused with the bilinear backward");
  m.def("status", &status, "read and clear the device error word (bounded-wait timeouts)");
}
