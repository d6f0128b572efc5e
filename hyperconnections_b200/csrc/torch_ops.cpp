// torch_ops.cpp — autograd Functions of the batched matrix exponentials in
// C++, over the C ABI of libhcops.so (include/hcops.h).
//
// The ops are tiny on the GPU (65,536 4x4 matrices forward + backward take
// about 29 us of kernels), so a Python autograd Function around ctypes calls
// spends several times that on the host (a ctypes call of eight arguments
// alone is ~5 us). Here the forward, the backward and their launches run in
// C++: the autograd engine calls the backward without entering Python.
// Semantics are those of hyperconnections_b200/ops/expm.py, which validates
// the arguments and calls these:
//   expm_t18(A, per_matrix)  T18 with global (or per-matrix) scaling; the
//                            forward's partial maxima of ||A||_1 stay in a
//                            buffer held by the graph for the backward (mode 2)
//   matrix_exp(A)            Pade [7/7] with per-matrix scaling
// A is float32-converted and made contiguous (no copy when it already is);
// results come back in A's shape and dtype.
#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <algorithm>

#include "../../include/hcops.h"

namespace {

using torch::autograd::AutogradContext;
using torch::autograd::tensor_list;

void check(int rc, const char* what) {
  TORCH_CHECK(rc == HC_OK, what, " failed: ", hc_error_string(rc), " (hcops status ", rc, ")");
}

torch::Tensor flat32(const torch::Tensor& A) {
  const int64_t n = A.size(-1);
  return A.to(torch::kFloat32).contiguous().view({-1, n, n});
}

void* stream_of(const torch::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

torch::Tensor restore(const torch::Tensor& t, c10::IntArrayRef sizes, c10::ScalarType dtype) {
  auto v = t.view(sizes);
  return dtype == torch::kFloat32 ? v : v.to(dtype);
}

struct ExpmT18 : public torch::autograd::Function<ExpmT18> {
  static torch::Tensor forward(AutogradContext* ctx, const torch::Tensor& A, bool per_matrix) {
    const c10::cuda::CUDAGuard guard(A.device());
    auto A32 = flat32(A);
    const int64_t batch = A32.size(0), n = A32.size(1), size = batch * n * n;
    torch::Tensor E, buf;
    float* scratch = nullptr;
    int64_t words = 0;
    if (per_matrix) {
      E = torch::empty_like(A32);
    } else {  // one allocation: E, then the partial maxima the backward reuses
      words = std::max<int64_t>(1, hc_expm_t18_scratch_words(batch, static_cast<int>(n)));
      buf = torch::empty({size + words}, A32.options());
      E = buf.narrow(0, 0, size).view({batch, n, n});
      scratch = buf.data_ptr<float>() + size;
    }
    check(hc_expm_t18_fwd(A32.data_ptr<float>(), E.data_ptr<float>(), batch, static_cast<int>(n), scratch, words,
                          per_matrix ? 1 : 0, stream_of(A32)),
          "hc_expm_t18_fwd");
    ctx->save_for_backward({A32});
    ctx->saved_data["buf"] = buf;
    ctx->saved_data["words"] = words;
    ctx->saved_data["per_matrix"] = per_matrix;
    ctx->saved_data["sizes"] = A.sizes().vec();
    ctx->saved_data["dtype"] = static_cast<int64_t>(A.scalar_type());
    return restore(E, A.sizes(), A.scalar_type());
  }

  static tensor_list backward(AutogradContext* ctx, tensor_list grads) {
    const auto A32 = ctx->get_saved_variables()[0];
    const c10::cuda::CUDAGuard guard(A32.device());
    const int64_t batch = A32.size(0), n = A32.size(1), size = batch * n * n;
    const bool per_matrix = ctx->saved_data["per_matrix"].toBool();
    const int64_t words = ctx->saved_data["words"].toInt();
    auto buf = ctx->saved_data["buf"].toTensor();
    float* scratch = buf.defined() ? buf.data_ptr<float>() + size : nullptr;
    auto G = grads[0].to(torch::kFloat32).contiguous().view({batch, n, n});
    auto dA = torch::empty_like(A32);
    check(hc_expm_t18_bwd(A32.data_ptr<float>(), G.data_ptr<float>(), dA.data_ptr<float>(), batch,
                          static_cast<int>(n), scratch, words, per_matrix ? 1 : 2, stream_of(A32)),
          "hc_expm_t18_bwd");
    const auto sizes = ctx->saved_data["sizes"].toIntVector();
    const auto dtype = static_cast<c10::ScalarType>(ctx->saved_data["dtype"].toInt());
    return {restore(dA, sizes, dtype), torch::Tensor()};
  }
};

struct MatrixExp : public torch::autograd::Function<MatrixExp> {
  static torch::Tensor forward(AutogradContext* ctx, const torch::Tensor& A) {
    const c10::cuda::CUDAGuard guard(A.device());
    auto A32 = flat32(A);
    const int64_t batch = A32.size(0), n = A32.size(1);
    auto E = torch::empty_like(A32);
    check(hc_expm_pade_fwd(A32.data_ptr<float>(), E.data_ptr<float>(), batch, static_cast<int>(n), stream_of(A32)),
          "hc_expm_pade_fwd");
    ctx->save_for_backward({A32});
    ctx->saved_data["sizes"] = A.sizes().vec();
    ctx->saved_data["dtype"] = static_cast<int64_t>(A.scalar_type());
    return restore(E, A.sizes(), A.scalar_type());
  }

  static tensor_list backward(AutogradContext* ctx, tensor_list grads) {
    const auto A32 = ctx->get_saved_variables()[0];
    const c10::cuda::CUDAGuard guard(A32.device());
    const int64_t batch = A32.size(0), n = A32.size(1);
    auto G = grads[0].to(torch::kFloat32).contiguous().view({batch, n, n});
    auto dA = torch::empty_like(A32);
    check(hc_expm_pade_bwd(A32.data_ptr<float>(), G.data_ptr<float>(), dA.data_ptr<float>(), batch,
                           static_cast<int>(n), stream_of(A32)),
          "hc_expm_pade_bwd");
    const auto sizes = ctx->saved_data["sizes"].toIntVector();
    const auto dtype = static_cast<c10::ScalarType>(ctx->saved_data["dtype"].toInt());
    return {restore(dA, sizes, dtype)};
  }
};

torch::Tensor expm_t18(const torch::Tensor& A, bool per_matrix) { return ExpmT18::apply(A, per_matrix); }
torch::Tensor matrix_exp(const torch::Tensor& A) { return MatrixExp::apply(A); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "autograd Functions of the batched matrix exponentials over libhcops.so";
  m.def("expm_t18", &expm_t18, "T18 matrix exponential (global or per-matrix scaling), differentiable");
  m.def("matrix_exp", &matrix_exp, "Pade [7/7] matrix exponential, differentiable");
  m.def("abi_version", &hc_abi_version, "ABI version of the linked libhcops.so");
}
