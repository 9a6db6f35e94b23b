// qrb200 -- PyTorch operator registration: torch.ops.qrb200.geqrf(A) -> (H, tau, info).
//
// The operator form of the reference entry point custom_kernel(data) -> (H, tau)
// (reflection_no_reflectors.py:181-196) for callers that dispatch through the torch operator
// registry (torch.ops, TorchScript, torch.compile graphs).  It is a thin layer over the C ABI of
// libqrb200.so (include/qrb200.h): no kernel lives here.
//   * A: (..., n, n) CUDA tensor of any floating dtype; float32 / bfloat16 / float16 are read
//     and written natively, others are converted to float32 first and the factors back, like
//     the reference's .to(float32) / .to(dtype) (:183, :196).
//   * H (..., n, n) and tau (..., n) in A's dtype, info (...) int32 QRB200_INFO_* bits.
//   * Enqueued on the current CUDA stream of A's device; the workspace comes from torch's
//     caching allocator.  A bad argument or a CUDA error raises (TORCH_CHECK).
// A Meta kernel gives shapes and dtypes without running anything.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "qrb200.h"

namespace {

bool native(at::ScalarType t) {
  return t == at::kFloat || t == at::kBFloat16 || t == at::kHalf;
}

int32_t dtype_code(at::ScalarType t) {
  return t == at::kFloat ? QRB200_F32 : (t == at::kBFloat16 ? QRB200_BF16 : QRB200_F16);
}

std::vector<int64_t> lead_sizes(const at::Tensor& A) {
  return std::vector<int64_t>(A.sizes().begin(), A.sizes().end() - 2);
}

void check_square(const at::Tensor& A) {
  TORCH_CHECK(A.dim() >= 2 && A.size(-1) == A.size(-2),
              "qrb200::geqrf expects a (..., n, n) tensor, got ", A.sizes());
  TORCH_CHECK(at::isFloatingType(A.scalar_type()), "qrb200::geqrf expects a floating dtype");
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> geqrf_cuda(const at::Tensor& data) {
  check_square(data);
  TORCH_CHECK(data.is_cuda(), "qrb200::geqrf: the CUDA kernel takes CUDA tensors");
  const c10::cuda::CUDAGuard guard(data.device());
  at::Tensor A = (native(data.scalar_type()) ? data : data.to(at::kFloat)).contiguous();
  const int64_t n = A.size(-1);
  auto lead = lead_sizes(A);
  int64_t batch = 1;
  for (int64_t d : lead) batch *= d;
  at::Tensor H = at::empty_like(A);
  auto tsz = lead;
  tsz.push_back(n);
  at::Tensor tau = at::empty(tsz, A.options());
  at::Tensor info = at::zeros(lead, A.options().dtype(at::kInt));
  if (batch > 0 && n > 0) {
    size_t ws_bytes = 0;
    int rc = qrb200_workspace_bytes(batch, (int32_t)n, &ws_bytes);
    TORCH_CHECK(rc == QRB200_OK, "qrb200_workspace_bytes: ", qrb200_status_string(rc));
    at::Tensor ws = at::empty({(int64_t)ws_bytes}, A.options().dtype(at::kByte));
    rc = qrb200_geqrf_batched(A.data_ptr(), H.data_ptr(), tau.data_ptr(),
                              info.data_ptr<int32_t>(), batch, (int32_t)n,
                              dtype_code(A.scalar_type()), ws_bytes ? ws.data_ptr() : nullptr,
                              ws_bytes, at::cuda::getCurrentCUDAStream().stream());
    TORCH_CHECK(rc == QRB200_OK, "qrb200_geqrf_batched: ", qrb200_status_string(rc),
                rc == QRB200_ERR_CUDA ? qrb200_last_cuda_error() : "");
  }
  if (!native(data.scalar_type())) {
    H = H.to(data.scalar_type());
    tau = tau.to(data.scalar_type());
  }
  return {H, tau, info};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> geqrf_meta(const at::Tensor& data) {
  check_square(data);
  auto lead = lead_sizes(data);
  auto tsz = lead;
  tsz.push_back(data.size(-1));
  return {at::empty_like(data), at::empty(tsz, data.options()),
          at::empty(lead, data.options().dtype(at::kInt))};
}

}  // namespace

TORCH_LIBRARY(qrb200, m) {
  m.def("geqrf(Tensor A) -> (Tensor H, Tensor tau, Tensor info)");
}

TORCH_LIBRARY_IMPL(qrb200, CUDA, m) { m.impl("geqrf", geqrf_cuda); }

TORCH_LIBRARY_IMPL(qrb200, Meta, m) { m.impl("geqrf", geqrf_meta); }
