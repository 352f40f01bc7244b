// Python bindings of the sm_100a kernel library.  Tensors are checked and translated into raw
// pointers/strides here; the CUDA translation units never include torch headers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <vector>

#include "common/host.h"
#include "attn/attn_api.h"
#include "gemm/api.h"
#include "gemm/ce_api.h"
#include "misc/rowops.h"
#include "comm/peer.h"
#include "optim/optim_api.h"
#include "misc/norm_variants.h"
#include "misc/spectral.h"

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

// Fused all-gather description from Python: None, or one tuple per staged B operand
// (src_ptrs [world], cuts [world + 1], done int32 [rows / 64], uses), where uses counts this gather
// among all gathers into that done array (1 for the first); the staging buffers are the weights
// passed as the B operands, dense [rows, cols] bf16.
bool make_gather(const py::object& obj, const std::vector<const Tensor*>& staging, ttb::gemm::Gather& g) {
  if (obj.is_none()) return false;
  const auto ops = obj.cast<std::vector<py::tuple>>();
  TORCH_CHECK(ops.size() == staging.size(), "gather: one description per staged operand");
  g = ttb::gemm::Gather{};
  g.nops = static_cast<int>(ops.size());
  g.claim = ttb::gather_claim_counter();
  for (size_t o = 0; o < ops.size(); ++o) {
    TORCH_CHECK(ops[o].size() == 4, "gather: (src_ptrs, cuts, done, uses)");
    const auto src = ops[o][0].cast<std::vector<int64_t>>();
    const auto cut = ops[o][1].cast<std::vector<int64_t>>();
    const Tensor done = ops[o][2].cast<Tensor>();
    const int64_t uses = ops[o][3].cast<int64_t>();
    TORCH_CHECK(uses >= 1, "gather: uses counts from 1");
    const Tensor& w = *staging[o];
    check_bf16(w, "gather staging");
    TORCH_CHECK(w.dim() == 2 && w.is_contiguous(), "gather staging must be a dense [rows, cols] matrix");
    const int64_t rows = w.size(0), cols = w.size(1);
    const int world = static_cast<int>(src.size());
    TORCH_CHECK(world >= 1 && world <= ttb::gemm::kGatherMaxRanks && cut.size() == src.size() + 1,
                "gather: 1..8 ranks and world + 1 cuts");
    TORCH_CHECK(rows % ttb::gemm::kGatherSlabRows == 0 && cols % 8 == 0, "gather: rows % 64 == 0 and cols % 8 == 0");
    TORCH_CHECK(cut[0] == 0 && cut[world] == rows, "gather: cuts must span the rows");
    for (int r = 0; r < world; ++r) {
      TORCH_CHECK(cut[r] <= cut[r + 1] && cut[r] % ttb::gemm::kGatherSlabRows == 0,
                  "gather: cuts ascend in 64-row steps");
      TORCH_CHECK(src[r] % 16 == 0, "gather: shard pointers must be 16-byte aligned");
      g.op[o].src[r] = reinterpret_cast<const __nv_bfloat16*>(src[r]);
      g.op[o].cut[r] = static_cast<int>(cut[r]);
    }
    g.op[o].cut[world] = static_cast<int>(rows);
    TORCH_CHECK(done.is_cuda() && done.scalar_type() == torch::kInt32 && done.is_contiguous() &&
                    done.numel() == rows / ttb::gemm::kGatherSlabRows && done.device() == w.device(),
                "gather: done must be int32 [rows / 64] on the staging buffer's device");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "gather: staging must be 16-byte aligned");
    g.op[o].world = world;
    g.op[o].rows = static_cast<int>(rows);
    g.op[o].cols = static_cast<int>(cols);
    g.op[o].dst = reinterpret_cast<__nv_bfloat16*>(w.data_ptr());
    g.op[o].done = reinterpret_cast<uint32_t*>(done.data_ptr<int>());
    g.op[o].target = static_cast<uint32_t>(uses * ttb::gemm::gather_chunks_per_slab(static_cast<int>(cols)));
  }
  TORCH_CHECK(g.nops == 1 || (g.op[0].rows == g.op[1].rows && g.op[0].cols == g.op[1].cols),
              "gather: two staged operands need equal shapes");
  return true;
}

void gather_rows(const Tensor& w, const py::object& gather) {
  const c10::cuda::CUDAGuard guard(w.device());
  ttb::gemm::Gather g;
  TORCH_CHECK(make_gather(gather, {&w}, g), "gather_rows needs a gather description");
  ttb::gather_rows(g, cur_stream());
}

// out = alpha * (a @ b + bias) + beta * c     (out/c: bf16 or fp32, row-major rows)
// With b2: out = alpha * (a @ cat(b, b2) + bias) + beta * c, the contraction concatenated in one pass.
// With gather, b must be the transpose view of a dense staging buffer w [N, K] (b = w.t()).
void mm(const Tensor& a, const Tensor& b, Tensor& out, const c10::optional<Tensor>& c, double alpha, double beta,
        const c10::optional<Tensor>& bias, const c10::optional<Tensor>& b2, int64_t tile_n, const py::object& gather) {
  const c10::cuda::CUDAGuard guard(a.device());
  const auto A = a_operand(a);
  const auto B = b_operand(b);
  const int M = a.size(0), K = a.size(1), N = b.size(1);
  ttb::Operand B2{};
  int k_split = 0;
  if (b2.has_value()) {
    B2 = b_operand(*b2);
    TORCH_CHECK(b2->size(1) == N && b.size(0) + b2->size(0) == K, "concatenated inner dimensions differ");
    TORCH_CHECK(B2.mn_major == B.mn_major, "concatenated B operands must share a layout");
    k_split = static_cast<int>(b.size(0));
    TORCH_CHECK(k_split % 64 == 0, "the first B operand's rows must be a multiple of 64");
  } else {
    TORCH_CHECK(b.size(0) == K, "inner dimensions differ");
  }
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
  ttb::gemm::Gather g;
  const Tensor w = b.t();
  const bool gathered = make_gather(gather, {&w}, g);
  TORCH_CHECK(!gathered || (!b2.has_value() && !B.mn_major), "gather: one K-major weight operand");
  ttb::gemm_linear(A, B, M, N, K, out.data_ptr(), out.stride(0), out.scalar_type() == torch::kFloat32, cp, ldc,
                   c_f32, static_cast<float>(alpha), static_cast<float>(beta), bp, cur_stream(),
                   b2.has_value() ? &B2 : nullptr, k_split, static_cast<int>(tile_n), gathered ? &g : nullptr);
}

// qkv = x w^T with the rotary embedding applied to the first rope_cols columns
Tensor qkv_rope(const Tensor& x, const Tensor& w, int64_t rope_cols, int64_t dk, const Tensor& pos,
                const Tensor& cos_t, const Tensor& sin_t, const c10::optional<Tensor>& norm_max,
                const py::object& gather) {
  const c10::cuda::CUDAGuard guard(x.device());
  const auto X = a_operand(x);
  const auto W = b_operand(w.t());
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "w shape");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && pos.is_contiguous() && pos.numel() == M, "pos int32 [M]");
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.is_contiguous() && cos_t.size(-1) == dk / 2, "cos table");
  TORCH_CHECK(sin_t.scalar_type() == torch::kFloat32 && sin_t.is_contiguous() && sin_t.sizes() == cos_t.sizes(),
              "sin table");
  unsigned int* nm = nullptr;
  if (norm_max.has_value()) {
    TORCH_CHECK(norm_max->scalar_type() == torch::kFloat32 && norm_max->is_contiguous() &&
                    norm_max->numel() == rope_cols / dk && norm_max->device() == x.device(),
                "norm_max: zeroed fp32 [rope_cols / dk] on the input's device");
    nm = reinterpret_cast<unsigned int*>(norm_max->data_ptr<float>());
  }
  ttb::gemm::Gather g;
  const bool gathered = make_gather(gather, {&w}, g);
  auto out = torch::empty({M, N}, x.options());
  ttb::gemm_qkv_rope(X, W, M, N, K, out.data_ptr(), out.stride(0), rope_cols, dk, pos.data_ptr<int>(),
                     cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), cur_stream(), nm, gathered ? &g : nullptr);
  return out;
}

// h = l*r (mode 0) / silu(l)*r (mode 1) with l = x wl^T (+bl), r = x wr^T (+br)
void bilinear(const Tensor& x, const Tensor& wl, const Tensor& wr, const c10::optional<Tensor>& bl,
              const c10::optional<Tensor>& br, int64_t mode, Tensor& h, const c10::optional<Tensor>& lo,
              const c10::optional<Tensor>& ro, const py::object& gather) {
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
  ttb::gemm::Gather g;
  const bool gathered = make_gather(gather, {&wl, &wr}, g);
  ttb::gemm_bilinear(X, WL, WR, M, N, K, h.data_ptr(), lp, rp, h.stride(0), blp, brp, static_cast<int>(mode),
                     cur_stream(), gathered ? &g : nullptr);
}

// dl, dr from dH = dy @ wd (wd: [d_out, N] weight of the down projection)
void bilinear_grad(const Tensor& dy, const Tensor& wd, const Tensor& l, const Tensor& r, Tensor& dl, Tensor& dr,
                   int64_t mode) {
  const c10::cuda::CUDAGuard guard(dy.device());
  const auto DY = a_operand(dy);
  const auto WD = b_operand(wd);
  const int M = dy.size(0), K = dy.size(1), N = wd.size(1);
  TORCH_CHECK(wd.size(0) == K, "wd shape");
  // l, r share one row stride, dl, dr another (dl, dr may be the two halves of one [M, 2N] buffer)
  for (const Tensor* t : std::initializer_list<const Tensor*>{&l, &r, &dl, &dr}) {
    check_bf16(*t, "bilinear factor");
    TORCH_CHECK(t->dim() == 2 && t->stride(1) == 1 && t->size(0) == M && t->size(1) == N, "factor shape");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "bilinear factors must be 16-byte aligned");
  }
  TORCH_CHECK(l.stride(0) == r.stride(0) && dl.stride(0) == dr.stride(0), "factor row strides");
  ttb::gemm_bilinear_grad(DY, WD, M, N, K, l.data_ptr(), r.data_ptr(), dl.data_ptr(), dr.data_ptr(), l.stride(0),
                          dl.stride(0), static_cast<int>(mode), cur_stream());
}


// ------------------------------------------------------------------ row ops
std::vector<Tensor> rmsnorm_fwd(const Tensor& x, const Tensor& w, int64_t groups, double eps) {
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.dim() == 2, "x: contiguous fp32 [N, d]");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.numel() == x.size(1), "w");
  const int N = x.size(0), d = x.size(1);
  auto y = torch::empty({N, d}, x.options().dtype(torch::kBFloat16));
  auto rstd = torch::empty({N, groups}, x.options());
  if (N > 0)
    ttb::rmsnorm_fwd(x.data_ptr<float>(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(), N, d, groups,
                     static_cast<float>(eps), cur_stream());
  return {y, rstd};
}

// dres (+)= dx; returns dw
Tensor rmsnorm_bwd(const Tensor& dy, const Tensor& x, const Tensor& w, const Tensor& rstd, Tensor& dres,
                   bool accumulate, int64_t groups, c10::optional<Tensor> out16, double scale16) {
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(dy.is_contiguous() && dy.sizes() == x.sizes(), "dy");
  TORCH_CHECK(dy.scalar_type() == torch::kFloat32 || dy.scalar_type() == torch::kBFloat16, "dy dtype");
  TORCH_CHECK(dres.scalar_type() == torch::kFloat32 && dres.is_contiguous() && dres.sizes() == x.sizes(), "dres");
  const int N = x.size(0), d = x.size(1);
  auto dw = torch::zeros({d}, x.options());
  if (N == 0) return dw;
  void* o16 = nullptr;
  if (out16.has_value()) {
    check_bf16(*out16, "out16");
    TORCH_CHECK(out16->is_contiguous() && out16->sizes() == x.sizes(), "out16: contiguous bf16 like x");
    o16 = out16->data_ptr();
  }
  auto part = torch::empty({ttb::rmsnorm_bwd_partials(N), d}, x.options());
  ttb::rmsnorm_bwd_ex(dy.data_ptr(), dy.scalar_type() == torch::kFloat32, x.data_ptr<float>(), w.data_ptr<float>(),
                      rstd.data_ptr<float>(), dres.data_ptr<float>(), accumulate, part.data_ptr<float>(),
                      dw.data_ptr<float>(), false, N, d, groups, o16, static_cast<float>(scale16), cur_stream());
  return dw;
}

void rope_(Tensor& buf, int64_t rope_cols, int64_t dk, const Tensor& pos, const Tensor& inv_freq, bool inverse) {
  const c10::cuda::CUDAGuard guard(buf.device());
  check_bf16(buf, "buf");
  TORCH_CHECK(buf.dim() == 2 && buf.stride(1) == 1, "buf rows");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && pos.is_contiguous() && pos.numel() == buf.size(0), "pos");
  TORCH_CHECK(inv_freq.scalar_type() == torch::kFloat32 && inv_freq.numel() == dk / 2, "inv_freq");
  if (buf.size(0) == 0) return;
  ttb::rope_apply(buf.data_ptr(), buf.stride(0), buf.size(0), rope_cols, dk, pos.data_ptr<int>(),
                  inv_freq.data_ptr<float>(), inverse, cur_stream());
}

Tensor embed_fwd(const Tensor& idx, const Tensor& W) {
  const c10::cuda::CUDAGuard guard(W.device());
  TORCH_CHECK(idx.scalar_type() == torch::kInt64 && idx.is_contiguous(), "idx: int64");
  TORCH_CHECK(W.scalar_type() == torch::kFloat32 && W.is_contiguous(), "W: fp32");
  auto x = torch::empty({idx.numel(), W.size(1)}, W.options());
  if (idx.numel() > 0)
    ttb::embed_fwd(reinterpret_cast<const long long*>(idx.data_ptr<int64_t>()), W.data_ptr<float>(), x.data_ptr<float>(), idx.numel(), W.size(1),
                   W.size(0), cur_stream());
  return x;
}

// dW += scatter of dx rows by idx, deterministic (stable sort by id)
void embed_bwd(const Tensor& idx, const Tensor& dx, Tensor& dW) {
  const c10::cuda::CUDAGuard guard(dW.device());
  TORCH_CHECK(dx.scalar_type() == torch::kFloat32 && dx.is_contiguous(), "dx: fp32");
  TORCH_CHECK(dW.scalar_type() == torch::kFloat32 && dW.is_contiguous(), "dW: fp32");
  if (idx.numel() == 0) return;
  auto sorted = torch::sort(idx.reshape({-1}), /*stable=*/true, 0, false);
  auto ids = std::get<0>(sorted).contiguous();
  auto order = std::get<1>(sorted).contiguous();
  ttb::embed_bwd(reinterpret_cast<const long long*>(ids.data_ptr<int64_t>()), reinterpret_cast<const long long*>(order.data_ptr<int64_t>()), dx.data_ptr<float>(), dW.data_ptr<float>(),
                 idx.numel(), dW.size(1), dW.size(0), cur_stream());
}

// ------------------------------------------------------------------ fused linear + CE
// returns (loss_rows [M] fp32, lse [M] fp32)
std::vector<Tensor> ce_fwd(const Tensor& x, const Tensor& w, int64_t V, double alpha, const Tensor& targets,
                           const c10::optional<Tensor>& zout) {
  const c10::cuda::CUDAGuard guard(x.device());
  const auto X = a_operand(x);
  const auto W = b_operand(w.t());
  const int M = x.size(0), K = x.size(1);
  TORCH_CHECK(w.size(1) == K && w.size(0) >= V, "w: [>=V, d]");
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && targets.is_contiguous() && targets.numel() == M, "targets");
  const int tiles = ttb::ce_num_tiles(V);
  auto opts = x.options().dtype(torch::kFloat32);
  auto pmax = torch::empty({M, tiles}, opts);
  auto psum = torch::empty({M, tiles}, opts);
  auto tlogit = torch::zeros({M}, opts);
  auto lse = torch::empty({M}, opts);
  auto loss = torch::empty({M}, opts);
  float* zp = nullptr;
  long long ldz = 0;
  int Npad = 0;
  if (zout.has_value()) {
    TORCH_CHECK(zout->scalar_type() == torch::kFloat32 && zout->dim() == 2 && zout->size(0) == M &&
                    zout->stride(1) == 1 && zout->size(1) >= V,
                "zout: fp32 [M, >=V] with unit column stride");
    zp = zout->data_ptr<float>();
    ldz = zout->stride(0);
    Npad = static_cast<int>(zout->size(1));
  }
  ttb::ce_forward(X, W, M, V, K, static_cast<float>(alpha), reinterpret_cast<const long long*>(targets.data_ptr<int64_t>()), pmax.data_ptr<float>(),
                  psum.data_ptr<float>(), tlogit.data_ptr<float>(), lse.data_ptr<float>(), loss.data_ptr<float>(),
                  cur_stream(), zp, ldz, Npad);
  return {loss, lse};
}

void ce_bwd_from_logits(const Tensor& z, double alpha, const Tensor& targets, const Tensor& lse, const Tensor& grad,
                        Tensor& dlogits) {
  const c10::cuda::CUDAGuard guard(z.device());
  TORCH_CHECK(z.scalar_type() == torch::kFloat32 && z.dim() == 2 && z.stride(1) == 1, "z: fp32 [M, Npad]");
  check_bf16(dlogits, "dlogits");
  const int M = z.size(0), Npad = z.size(1);
  TORCH_CHECK(dlogits.dim() == 2 && dlogits.size(0) == M && dlogits.size(1) == Npad && dlogits.stride(1) == 1,
              "dlogits: bf16 [M, Npad]");
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && targets.is_contiguous() && targets.numel() == M, "targets");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() && lse.numel() == M, "lse");
  TORCH_CHECK(grad.scalar_type() == torch::kFloat32 && grad.numel() == 1, "grad: fp32 scalar");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(z.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(dlogits.data_ptr()) % 8 == 0,
              "alignment");
  ttb::ce_backward_from_logits(z.data_ptr<float>(), z.stride(0), M, Npad, static_cast<float>(alpha),
                               reinterpret_cast<const long long*>(targets.data_ptr<int64_t>()), lse.data_ptr<float>(),
                               grad.data_ptr<float>(), dlogits.data_ptr(), dlogits.stride(0), cur_stream());
}

void ce_bwd_logits(const Tensor& x, const Tensor& w, int64_t V, double alpha, const Tensor& targets, const Tensor& lse,
                   const Tensor& grad, Tensor& dlogits) {
  const c10::cuda::CUDAGuard guard(x.device());
  const auto X = a_operand(x);
  const auto W = b_operand(w.t());
  const int M = x.size(0), K = x.size(1);
  check_bf16(dlogits, "dlogits");
  TORCH_CHECK(dlogits.dim() == 2 && dlogits.size(0) == M && dlogits.stride(1) == 1, "dlogits");
  TORCH_CHECK(grad.scalar_type() == torch::kFloat32 && grad.numel() == 1, "grad: fp32 scalar");
  const int Npad = dlogits.size(1);
  TORCH_CHECK(w.size(0) >= Npad, "w rows must cover the padded logits");
  ttb::ce_backward_logits(X, W, M, Npad, V, K, static_cast<float>(alpha), reinterpret_cast<const long long*>(targets.data_ptr<int64_t>()),
                          lse.data_ptr<float>(), grad.data_ptr<float>(), dlogits.data_ptr(), dlogits.stride(0),
                          cur_stream());
}

// ------------------------------------------------------------------ polynomial attention
ttb::attn::Params attn_params(const std::vector<int64_t>& cols, const Tensor& pos, const Tensor& doc,
                              const Tensor& row_scale, const Tensor& par, int64_t B, int64_t T, int64_t H, int64_t dk) {
  TORCH_CHECK(cols.size() == 5, "cols: q1,k1,q2,k2,v offsets");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && pos.is_contiguous() && pos.numel() == B * T, "pos int32 [B*T]");
  TORCH_CHECK(doc.scalar_type() == torch::kInt32 && doc.is_contiguous() && doc.numel() == B * T, "doc int32 [B*T]");
  TORCH_CHECK(row_scale.scalar_type() == torch::kFloat32 && row_scale.is_contiguous() && row_scale.numel() == B * T,
              "row_scale fp32 [B*T]");
  TORCH_CHECK(par.scalar_type() == torch::kFloat32 && par.is_contiguous() && par.numel() == H * 4, "par fp32 [H,4]");
  for (auto c : cols) TORCH_CHECK(c % 64 == 0, "projection column offsets must be multiples of 64");
  ttb::attn::Params p{};
  p.B = B; p.T = T; p.H = H;
  p.cq1 = cols[0]; p.ck1 = cols[1]; p.cq2 = cols[2]; p.ck2 = cols[3]; p.cv = cols[4];
  p.pos = pos.data_ptr<int>();
  p.doc = doc.data_ptr<int>();
  p.row_scale = row_scale.data_ptr<float>();
  p.par = par.data_ptr<float>();
  p.sm = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dk)));
  return p;
}

Tensor poly_fwd(int64_t kind, int64_t dk, int64_t dv, const Tensor& qkv, std::vector<int64_t> cols, const Tensor& pos,
                const Tensor& doc, const Tensor& row_scale, const Tensor& par, int64_t B, int64_t T, int64_t H) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  check_bf16(qkv, "qkv");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(0) == B * T, "qkv [B*T, ld]");
  auto p = attn_params(cols, pos, doc, row_scale, par, B, T, H, dk);
  auto y = torch::empty({B * T, H * dv}, qkv.options());
  p.y = static_cast<__nv_bfloat16*>(y.data_ptr());
  p.ldy = y.stride(0);
  ttb::poly_attention_fwd(kind, dk, dv, qkv.data_ptr(), qkv.stride(0), p, cur_stream());
  return y;
}

// returns (dqkv [B*T, ld] bf16 in the qkv layout, dpar [B*H, blocks, 4] fp32)
std::vector<Tensor> poly_bwd(int64_t kind, int64_t dk, int64_t dv, const Tensor& qkv, std::vector<int64_t> cols,
                             const Tensor& dout, const Tensor& pos, const Tensor& doc, const Tensor& doc_end,
                             const Tensor& row_scale, const Tensor& par, int64_t B, int64_t T, int64_t H,
                             const c10::optional<Tensor>& rope_cos, const c10::optional<Tensor>& rope_sin) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  check_bf16(qkv, "qkv");
  check_bf16(dout, "dout");
  TORCH_CHECK(dout.dim() == 2 && dout.stride(1) == 1 && dout.size(0) == B * T && dout.size(1) == H * dv, "dout");
  TORCH_CHECK(doc_end.scalar_type() == torch::kInt32 && doc_end.is_contiguous() && doc_end.numel() == B * T, "doc_end");
  auto p = attn_params(cols, pos, doc, row_scale, par, B, T, H, dk);
  // every element of dqkv is written by the two kernels (all rows < B*T, all five column groups)
  auto dqkv = torch::empty_like(qkv);
  const int blocks = ttb::poly_attention_dpar_blocks(T);
  if (rope_cos.has_value()) {
    TORCH_CHECK(rope_sin.has_value(), "rope tables come in pairs");
    TORCH_CHECK(rope_cos->scalar_type() == torch::kFloat32 && rope_cos->is_contiguous() && rope_cos->size(-1) == dk / 2,
                "rope cos table [positions, dk/2]");
    TORCH_CHECK(rope_sin->sizes() == rope_cos->sizes() && rope_sin->is_contiguous(), "rope sin table");
    p.rope_cos = rope_cos->data_ptr<float>();
    p.rope_sin = rope_sin->data_ptr<float>();
  }
  auto dpar = torch::zeros({B * H, blocks, 4}, qkv.options().dtype(torch::kFloat32));
  p.dq = static_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.ldd = dqkv.stride(0);
  p.dpar = dpar.data_ptr<float>();
  ttb::poly_attention_bwd(kind, dk, dv, qkv.data_ptr(), qkv.stride(0), dout.data_ptr(), dout.stride(0),
                          doc_end.data_ptr<int>(), p, cur_stream());
  return {dqkv, dpar};
}

// ---------------------------------------------------------------------------- peer collectives
ttb::PeerPtrs peer_ptrs(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(!ptrs.empty() && static_cast<int>(ptrs.size()) <= ttb::kMaxPeers, "1..8 peer pointers");
  ttb::PeerPtrs p{};
  for (size_t i = 0; i < ptrs.size(); ++i) p.p[i] = reinterpret_cast<void*>(ptrs[i]);
  return p;
}

void peer_barrier(const std::vector<int64_t>& pads, int64_t rank, int64_t epoch, int64_t limit_cycles) {
  ttb::peer_barrier(peer_ptrs(pads), static_cast<int>(pads.size()), static_cast<int>(rank),
                    static_cast<uint32_t>(epoch), limit_cycles, cur_stream());
}

// Pull-based reduce-scatter of the flat fp32 buffers: out (this rank's region of its own buffer)
// = sum over ranks of their [off, off + n); returns the per-block partial sums of squares (fp64).
Tensor rs_reduce_sq(const std::vector<int64_t>& bufs, int64_t off, Tensor& out) {
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous(), "out: contiguous fp32");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out: 16-byte aligned");
  auto partial = torch::empty({ttb::rs_reduce_blocks()}, out.options().dtype(torch::kFloat64));
  ttb::rs_reduce_sq(peer_ptrs(bufs), static_cast<int>(bufs.size()), off, out.numel(), out.data_ptr<float>(),
                    partial.data_ptr<double>(), false, 0, cur_stream());
  return partial;
}

// out += sum over ranks of bufs[q][off : off + out.numel()] (rank order, deterministic).
void rs_accumulate(const std::vector<int64_t>& bufs, int64_t off, Tensor& out, int64_t blocks) {
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous(), "out: contiguous fp32");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out: 16-byte aligned");
  ttb::rs_reduce_sq(peer_ptrs(bufs), static_cast<int>(bufs.size()), off, out.numel(), out.data_ptr<float>(),
                    nullptr, true, static_cast<int>(blocks), cur_stream());
}

// segs: int64 [nseg, 4] rows (src, dst32, dst16, n) of device addresses (0 = absent), on the device.
void ag_pull_cast(const Tensor& segs, int64_t max_n) {
  TORCH_CHECK(segs.scalar_type() == torch::kInt64 && segs.is_cuda() && segs.is_contiguous() && segs.dim() == 2 &&
                  segs.size(1) == 4,
              "segs: int64 [nseg, 4] on the device");
  static_assert(sizeof(ttb::CopySeg) == 32, "CopySeg layout");
  ttb::ag_pull_cast(reinterpret_cast<const ttb::CopySeg*>(segs.data_ptr<int64_t>()), static_cast<int>(segs.size(0)),
                    max_n, cur_stream());
}

int64_t status() { return static_cast<int64_t>(ttb::status_read_and_reset()); }

// ------------------------------------------------------------------------------------ optimizer
const float* scale_ptr(const c10::optional<Tensor>& grad_scale) {
  if (!grad_scale.has_value()) return nullptr;
  TORCH_CHECK(grad_scale->is_cuda() && grad_scale->scalar_type() == torch::kFloat32 && grad_scale->numel() == 1,
              "grad_scale: one fp32 element on the device");
  return grad_scale->data_ptr<float>();
}

void check_matrix_f32(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kFloat32 && t.dim() == 2 && t.is_contiguous(), name,
              " must be a contiguous 2-D fp32 tensor");
}

// table: int64 [count, 8] device rows (p, g, exp_avg, exp_avg_sq, step, cache, n, first_chunk).
void adamw_update(const Tensor& table, int64_t total_chunks, double lr, double beta1, double beta2, double eps,
                  double weight_decay, const c10::optional<Tensor>& grad_scale) {
  check_cuda(table, "table");
  TORCH_CHECK(table.scalar_type() == torch::kInt64 && table.dim() == 2 && table.size(1) == 8 && table.is_contiguous(),
              "table: contiguous int64 [count, 8]");
  const c10::cuda::CUDAGuard guard(table.device());
  ttb::adamw_update(reinterpret_cast<const ttb::AdamwTensor*>(table.data_ptr()), static_cast<int>(table.size(0)),
                    total_chunks, static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2),
                    static_cast<float>(eps), static_cast<float>(weight_decay), scale_ptr(grad_scale), cur_stream());
}

// Returns the number of partial sums written into `partial`.
int64_t muon_prepare(const Tensor& g, Tensor& buf, Tensor& x, Tensor& partial, double w_buf, double w_nesterov,
                     bool nesterov, bool transpose, const c10::optional<Tensor>& grad_scale) {
  check_matrix_f32(g, "g");
  check_matrix_f32(buf, "buf");
  check_bf16(x, "x");
  TORCH_CHECK(buf.sizes() == g.sizes(), "buf must match g");
  const int rows = g.size(0), cols = g.size(1);
  TORCH_CHECK(x.is_contiguous() && x.dim() == 2 && x.size(0) == (transpose ? cols : rows) &&
                  x.size(1) == (transpose ? rows : cols), "x: contiguous, g's shape (transposed if asked)");
  TORCH_CHECK(partial.is_cuda() && partial.scalar_type() == torch::kFloat32 && partial.numel() >= ttb::kMuonMaxPartials,
              "partial: fp32 with room for the partial sums");
  const c10::cuda::CUDAGuard guard(g.device());
  return ttb::muon_prepare(g.data_ptr<float>(), buf.data_ptr<float>(),
                           reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), partial.data_ptr<float>(), rows, cols,
                           static_cast<float>(w_buf), static_cast<float>(w_nesterov), nesterov, transpose,
                           scale_ptr(grad_scale), cur_stream());
}

void muon_normalize(Tensor& x, const Tensor& partial, int64_t n_partial, double eps) {
  check_bf16(x, "x");
  TORCH_CHECK(x.is_contiguous(), "x must be contiguous");
  TORCH_CHECK(partial.is_cuda() && partial.scalar_type() == torch::kFloat32 && partial.numel() >= n_partial,
              "partial: fp32 holding n_partial sums");
  const c10::cuda::CUDAGuard guard(x.device());
  ttb::muon_normalize(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.numel(), partial.data_ptr<float>(),
                      static_cast<int>(n_partial), static_cast<float>(eps), cur_stream());
}

// p = p * decay + alpha * o (o: p's shape, or transposed); cache (optional bf16 [rows, cols] view with
// unit column stride) receives bf16(p).
void muon_apply(Tensor& p, const Tensor& o, bool transposed, double decay, double alpha,
                const c10::optional<Tensor>& cache) {
  check_matrix_f32(p, "p");
  check_bf16(o, "o");
  const int rows = p.size(0), cols = p.size(1);
  TORCH_CHECK(o.is_contiguous() && o.dim() == 2 && o.size(0) == (transposed ? cols : rows) &&
                  o.size(1) == (transposed ? rows : cols), "o: contiguous, p's shape (transposed if so flagged)");
  __nv_bfloat16* c = nullptr;
  int64_t ld = 0;
  if (cache.has_value()) {
    check_bf16(*cache, "cache");
    TORCH_CHECK(cache->dim() == 2 && cache->size(0) == rows && cache->size(1) == cols && cache->stride(1) == 1,
                "cache: bf16 [rows, cols] with unit column stride");
    c = reinterpret_cast<__nv_bfloat16*>(cache->data_ptr());
    ld = cache->stride(0);
  }
  const c10::cuda::CUDAGuard guard(p.device());
  ttb::muon_apply(p.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), rows, cols, transposed,
                  static_cast<float>(decay), static_cast<float>(alpha), c, ld, cur_stream());
}

// ------------------------------------------------------------------------------------ norm variants
ttb::NormVariantArgs nv_args(const Tensor& x, const Tensor& w, const c10::optional<Tensor>& w2, int64_t mode,
                             double g, double b, const c10::optional<Tensor>& a_dev, double eps) {
  check_matrix_f32(x, "x");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.numel() == x.size(1),
              "w: contiguous fp32 [d]");
  ttb::NormVariantArgs a{};
  a.mode = static_cast<int>(mode);
  a.N = x.size(0);
  a.d = x.size(1);
  a.eps = static_cast<float>(eps);
  a.g = static_cast<float>(g);
  a.b = static_cast<float>(b);
  a.w = w.data_ptr<float>();
  if (w2.has_value()) {
    TORCH_CHECK(w2->is_cuda() && w2->scalar_type() == torch::kFloat32 && w2->is_contiguous() &&
                    w2->numel() == x.size(1), "w2: contiguous fp32 [d]");
    a.w2 = w2->data_ptr<float>();
  }
  if (a_dev.has_value()) {
    TORCH_CHECK(a_dev->is_cuda() && a_dev->scalar_type() == torch::kFloat32 && a_dev->numel() == 1,
                "scale: one fp32 element on the device");
    a.a_dev = a_dev->data_ptr<float>();
  }
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(a.w) % 16 == 0 &&
                  (a.w2 == nullptr || reinterpret_cast<uintptr_t>(a.w2) % 16 == 0), "x, w, w2: 16-byte aligned");
  return a;
}

// Returns [y16, y32, r, msq]; an output not asked for is an empty tensor.
std::vector<Tensor> norm_variant_fwd(const Tensor& x, const Tensor& w, const c10::optional<Tensor>& w2, int64_t mode,
                                     double g, double b, const c10::optional<Tensor>& a_dev, double eps, bool want16,
                                     bool want32, const c10::optional<Tensor>& resid, double alpha, bool want_r,
                                     bool want_msq) {
  const auto a = nv_args(x, w, w2, mode, g, b, a_dev, eps);
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor y16, y32, r, msq;
  if (want16) y16 = torch::empty({a.N, a.d}, x.options().dtype(torch::kBFloat16));
  if (want32) y32 = torch::empty({a.N, a.d}, x.options());
  if (want_r) r = torch::empty({a.N}, x.options());
  if (want_msq) msq = torch::empty({a.N}, x.options());
  const float* res = nullptr;
  if (resid.has_value()) {
    TORCH_CHECK(want32, "a residual needs the fp32 result");
    check_matrix_f32(*resid, "resid");
    TORCH_CHECK(resid->sizes() == x.sizes(), "resid must match x");
    res = resid->data_ptr<float>();
  }
  ttb::norm_variant_fwd(a, x.data_ptr<float>(), res, static_cast<float>(alpha), want16 ? y16.data_ptr() : nullptr,
                        want32 ? y32.data_ptr<float>() : nullptr, want_r ? r.data_ptr<float>() : nullptr,
                        want_msq ? msq.data_ptr<float>() : nullptr, cur_stream());
  return {y16, y32, r, msq};
}

// Returns [dx, dw, dw2]; dx is `dx_out` (added to when accumulate) or a new tensor.
std::vector<Tensor> norm_variant_bwd(const Tensor& dy, const Tensor& x, const Tensor& w,
                                     const c10::optional<Tensor>& w2, int64_t mode, double g, double b,
                                     const c10::optional<Tensor>& a_dev, double eps, double dy_scale,
                                     const c10::optional<Tensor>& r, const c10::optional<Tensor>& dr,
                                     const c10::optional<Tensor>& dx_out, bool accumulate, bool want_dw,
                                     bool want_dw2) {
  const auto a = nv_args(x, w, w2, mode, g, b, a_dev, eps);
  check_cuda(dy, "dy");
  TORCH_CHECK(dy.is_contiguous() && dy.sizes() == x.sizes() &&
                  (dy.scalar_type() == torch::kFloat32 || dy.scalar_type() == torch::kBFloat16),
              "dy: contiguous fp32 or bf16 of x's shape");
  const float* rp = nullptr;
  const float* drp = nullptr;
  if (r.has_value()) {
    TORCH_CHECK(r->is_cuda() && r->scalar_type() == torch::kFloat32 && r->numel() == a.N, "r: fp32 [N]");
    rp = r->data_ptr<float>();
  }
  if (dr.has_value()) {
    TORCH_CHECK(dr->is_cuda() && dr->scalar_type() == torch::kFloat32 && dr->numel() == a.N &&
                    dr->is_contiguous(), "dr: contiguous fp32 [N]");
    drp = dr->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor dx;
  if (dx_out.has_value()) {
    check_matrix_f32(*dx_out, "dx");
    TORCH_CHECK(dx_out->sizes() == x.sizes(), "dx must match x");
    dx = *dx_out;
  } else {
    TORCH_CHECK(!accumulate, "accumulating needs a dx buffer");
    dx = torch::empty_like(x);
  }
  Tensor dw, dw2, part;
  if (want_dw) dw = torch::empty({a.d}, x.options());
  if (want_dw2) dw2 = torch::empty({a.d}, x.options());
  if (want_dw || want_dw2)
    part = torch::empty({(want_dw2 ? 2 : 1) * static_cast<int64_t>(ttb::norm_variant_partials(a.N)) * a.d}, x.options());
  ttb::norm_variant_bwd(a, dy.data_ptr(), dy.scalar_type() == torch::kFloat32, static_cast<float>(dy_scale),
                        x.data_ptr<float>(), rp, drp, dx.data_ptr<float>(), accumulate,
                        want_dw ? dw.data_ptr<float>() : nullptr, want_dw2 ? dw2.data_ptr<float>() : nullptr,
                        part.defined() ? part.data_ptr<float>() : nullptr, cur_stream());
  return {dx, dw, dw2};
}

// ------------------------------------------------------------------------------------ spectral linear
void check_vec_f32(const Tensor& t, int64_t n, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kFloat32 && t.is_contiguous() && t.numel() == n, name,
              ": contiguous fp32 with the expected length");
}

Tensor spectral_scratch(const Tensor& w) {
  return torch::empty({ttb::spectral_scratch_floats(w.size(0), w.size(1))}, w.options());
}

// Writes bf16(gamma W / max(|sigma|, floor)) into out (bf16 [rows, cols], unit column stride);
// returns sigma = u^T W v (fp32 [1]).
Tensor spectral_cast(const Tensor& w, const Tensor& gamma, const Tensor& u, const Tensor& v, double floor_,
                     Tensor& out) {
  check_matrix_f32(w, "weight");
  const int rows = w.size(0), cols = w.size(1);
  check_vec_f32(gamma, 1, "gamma");
  check_vec_f32(u, rows, "u");
  check_vec_f32(v, cols, "v");
  check_bf16(out, "out");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == rows && out.size(1) == cols && out.stride(1) == 1 &&
                  out.stride(0) % 4 == 0, "out: bf16 [rows, cols], unit column stride, row stride a multiple of 4");
  const c10::cuda::CUDAGuard guard(w.device());
  auto sigma = torch::empty({1}, w.options());
  auto scratch = spectral_scratch(w);
  ttb::spectral_cast(w.data_ptr<float>(), rows, cols, gamma.data_ptr<float>(), u.data_ptr<float>(),
                     v.data_ptr<float>(), static_cast<float>(floor_), sigma.data_ptr<float>(),
                     scratch.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0),
                     cur_stream());
  return sigma;
}

// Returns [dW, dgamma] from dW_eff (fp32 [rows, cols], unit column stride).
std::vector<Tensor> spectral_grad(const Tensor& dwe, const Tensor& w, const Tensor& gamma, const Tensor& u,
                                  const Tensor& v, const Tensor& sigma, double floor_) {
  check_matrix_f32(w, "weight");
  const int rows = w.size(0), cols = w.size(1);
  check_cuda(dwe, "dW_eff");
  TORCH_CHECK(dwe.scalar_type() == torch::kFloat32 && dwe.dim() == 2 && dwe.size(0) == rows && dwe.size(1) == cols &&
                  dwe.stride(1) == 1, "dW_eff: fp32 [rows, cols] with unit column stride");
  check_vec_f32(gamma, 1, "gamma");
  check_vec_f32(u, rows, "u");
  check_vec_f32(v, cols, "v");
  check_vec_f32(sigma, 1, "sigma");
  const c10::cuda::CUDAGuard guard(w.device());
  auto dw = torch::empty_like(w);
  auto dgamma = torch::empty({1}, w.options());
  auto scratch = spectral_scratch(w);
  ttb::spectral_grad(dwe.data_ptr<float>(), dwe.stride(0), w.data_ptr<float>(), rows, cols, gamma.data_ptr<float>(),
                     u.data_ptr<float>(), v.data_ptr<float>(), sigma.data_ptr<float>(), static_cast<float>(floor_),
                     scratch.data_ptr<float>(), dw.data_ptr<float>(), dgamma.data_ptr<float>(), cur_stream());
  return {dw, dgamma};
}

void spectral_power_step(const Tensor& w, Tensor& u, Tensor& v, double floor_) {
  check_matrix_f32(w, "weight");
  check_vec_f32(u, w.size(0), "u");
  check_vec_f32(v, w.size(1), "v");
  const c10::cuda::CUDAGuard guard(w.device());
  auto scratch = spectral_scratch(w);
  ttb::spectral_power_step(w.data_ptr<float>(), w.size(0), w.size(1), u.data_ptr<float>(), v.data_ptr<float>(),
                           static_cast<float>(floor_), scratch.data_ptr<float>(), cur_stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tensor_train_ing_b200 sm_100a kernels (tcgen05 / TMEM / TMA)";
  m.def("mm", &mm, "out = alpha*(a@b + bias) + beta*c on the tcgen05 GEMM", py::arg("a"), py::arg("b"),
        py::arg("out"), py::arg("c") = py::none(), py::arg("alpha") = 1.0, py::arg("beta") = 0.0,
        py::arg("bias") = py::none(), py::arg("b2") = py::none(), py::arg("tile_n") = 0,
        py::arg("gather") = py::none());
  m.def("bilinear", &bilinear, "dual-B GEMM forming the bilinear hidden layer", py::arg("x"), py::arg("wl"),
        py::arg("wr"), py::arg("bl"), py::arg("br"), py::arg("mode"), py::arg("h"), py::arg("lo"), py::arg("ro"),
        py::arg("gather") = py::none());
  m.def("gather_rows", &gather_rows, "copy a row-sharded weight into its staging buffer (the fused GEMM's gather "
        "without the GEMM)", py::arg("w"), py::arg("gather"));
  m.def("bilinear_grad", &bilinear_grad, "dH GEMM fused with the bilinear backward");
  m.def("status", &status, "read and clear the device error word (bounded-wait timeouts)");
  m.def("peer_barrier", &peer_barrier, "cross-GPU barrier through symmetric signal pads (bounded wait)",
        py::arg("pads"), py::arg("rank"), py::arg("epoch"), py::arg("limit_cycles") = 2000000000LL);
  m.def("rs_accumulate", &rs_accumulate, "pull reduction over peer buffers added into a local accumulator",
        py::arg("bufs"), py::arg("off"), py::arg("out"), py::arg("blocks") = 0);
  m.def("rs_reduce_sq", &rs_reduce_sq, "pull reduce-scatter over peer buffers with fused sum-of-squares partials");
  m.def("ag_pull_cast", &ag_pull_cast, "pull all-gather over peer buffers with fused bf16 weight-cache writes");
  m.def("rmsnorm_fwd", &rmsnorm_fwd, "(group) RMSNorm: fp32 x -> bf16 y, fp32 rstd");
  m.def("rmsnorm_bwd", &rmsnorm_bwd, "(group) RMSNorm backward; adds dx into the residual grad, returns dw",
        py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dres"), py::arg("accumulate"),
        py::arg("groups"), py::arg("out16") = py::none(), py::arg("scale16") = 1.0);
  m.def("rope_", &rope_, "in-place rotary embedding (or its inverse) on a bf16 [N, ld] buffer");
  m.def("embed_fwd", &embed_fwd, "fp32 embedding gather");
  m.def("embed_bwd", &embed_bwd, "deterministic embedding backward (accumulates into dW)");
  m.def("ce_fwd", &ce_fwd, "fused linear + cross-entropy forward: per-row loss and lse", py::arg("x"), py::arg("w"),
        py::arg("V"), py::arg("alpha"), py::arg("targets"), py::arg("zout") = py::none());
  m.def("ce_bwd_from_logits", &ce_bwd_from_logits, "softmax-grad dlogits from the logits the forward kept");
  m.def("ce_bwd_logits", &ce_bwd_logits, "fused logits recompute + softmax-grad epilogue");
  m.def("poly_fwd", &poly_fwd, "tcgen05 polynomial attention forward");
  m.def("attn_grid_limit", [](int64_t limit) { ttb::poly_attention_set_grid_limit(static_cast<int>(limit)); },
        "cap the CTA count of the persistent attention kernels (0 = one per SM)");
  m.def("poly_bwd", &poly_bwd, "tcgen05 polynomial attention backward (dq and dkv kernels)", py::arg("kind"),
        py::arg("dk"), py::arg("dv"), py::arg("qkv"), py::arg("cols"), py::arg("dout"), py::arg("pos"), py::arg("doc"),
        py::arg("doc_end"), py::arg("row_scale"), py::arg("par"), py::arg("B"), py::arg("T"), py::arg("H"),
        py::arg("rope_cos") = py::none(), py::arg("rope_sin") = py::none());
  m.def("adamw_update", &adamw_update, "multi-tensor AdamW step (step counters, clip scale, bf16 copies)",
        py::arg("table"), py::arg("total_chunks"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"),
        py::arg("weight_decay"), py::arg("grad_scale") = py::none());
  m.def("muon_prepare", &muon_prepare, "Muon momentum + Nesterov + bf16 operand + sum of squares",
        py::arg("g"), py::arg("buf"), py::arg("x"), py::arg("partial"), py::arg("w_buf"), py::arg("w_nesterov"),
        py::arg("nesterov"), py::arg("transpose"), py::arg("grad_scale") = py::none());
  m.def("muon_normalize", &muon_normalize, "divide the Newton-Schulz operand by its bf16 Frobenius norm");
  m.def("muon_apply", &muon_apply, "Muon decay + update + bf16 weight copy", py::arg("p"), py::arg("o"),
        py::arg("transposed"), py::arg("decay"), py::arg("alpha"), py::arg("cache") = py::none());
  m.def("norm_variant_fwd", &norm_variant_fwd, "lagged / taper / fp32-output RMS row normalisation",
        py::arg("x"), py::arg("w"), py::arg("w2"), py::arg("mode"), py::arg("g"), py::arg("b"), py::arg("scale"),
        py::arg("eps"), py::arg("want16"), py::arg("want32"), py::arg("resid"), py::arg("alpha"), py::arg("want_r"),
        py::arg("want_msq"));
  m.def("norm_variant_bwd", &norm_variant_bwd, "backward of norm_variant_fwd (dx, dw, dw2)", py::arg("dy"),
        py::arg("x"), py::arg("w"), py::arg("w2"), py::arg("mode"), py::arg("g"), py::arg("b"), py::arg("scale"),
        py::arg("eps"), py::arg("dy_scale"), py::arg("r"), py::arg("dr"), py::arg("dx"), py::arg("accumulate"),
        py::arg("want_dw"), py::arg("want_dw2"));
  m.def("spectral_cast", &spectral_cast, "sigma = u^T W v and the bf16 effective weight");
  m.def("spectral_grad", &spectral_grad, "dW and dgamma of the spectral effective weight");
  m.def("spectral_power_step", &spectral_power_step, "one power-iteration step on u and v");
  m.def("qkv_rope", &qkv_rope, "QKV projection GEMM with the rotary embedding in its epilogue (optionally the "
        "per-head maximum row norms)", py::arg("x"), py::arg("w"), py::arg("rope_cols"), py::arg("dk"), py::arg("pos"),
        py::arg("cos_t"), py::arg("sin_t"), py::arg("norm_max") = py::none(), py::arg("gather") = py::none());
}
