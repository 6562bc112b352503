// Torch bindings for the sm_100a kernel library. The .cu files expose a plain C ABI (no torch
// headers, so they compile quickly and can be linked from non-torch hosts); this file adapts
// torch tensors to it and checks shapes, dtypes and alignment before any launch.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "api.h"

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_DT(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has wrong dtype")
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).dim() >= 1 && (x).stride(-1) == 1, #x " must have unit inner stride")

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

static void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed with code ", rc);
}

// ------------------------------------------------------------------ GEMM
// a: stored 2-D [a_rows, a_cols]; b: stored 2-D [b_rows, b_cols]; c: output buffer (any shape,
// row stride ldc). See gemm_sm100.cu for the modes.
void gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor c, int64_t M,
          int64_t N, int64_t K, int64_t mode, c10::optional<torch::Tensor> group_offsets,
          int64_t num_groups, int64_t b_rows_per_group, int64_t c_group_stride, int64_t epi,
          double alpha, int64_t bn, torch::Tensor err) {
  CHECK_CUDA(a); CHECK_CUDA(b); CHECK_CUDA(c);
  CHECK_DT(a, at::kBFloat16); CHECK_DT(b, at::kBFloat16);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "gemm operands must be 2-D views");
  CHECK_ROWMAJOR(a); CHECK_ROWMAJOR(b); CHECK_ROWMAJOR(c);
  TORCH_CHECK((epi & 1) ? c.scalar_type() == at::kFloat : c.scalar_type() == at::kBFloat16,
              "output dtype does not match epilogue");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "row strides must be 16-byte multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0, "operands must be 16-byte aligned");
  TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8");
  const int64_t ldc = c.dim() >= 2 ? c.stride(-2) : N;
  TORCH_CHECK(ldc % 8 == 0 || (epi & 1), "ldc must be a multiple of 8");
  const int* go = nullptr;
  if (mode != 0) {
    TORCH_CHECK(group_offsets.has_value(), "grouped modes need group_offsets");
    CHECK_DT(group_offsets.value(), at::kInt);
    go = group_offsets.value().data_ptr<int>();
  }
  c10::cuda::CUDAGuard g(a.device());
  int rc = mb_gemm_bf16(a.data_ptr(), a.size(0), a.size(1), a.stride(0), a_mn, b.data_ptr(),
                        b.size(0), b.size(1), b.stride(0), b_mn, c.data_ptr(), ldc, (int)M, (int)N,
                        (int)K, (int)mode, go, (int)num_groups, (int)b_rows_per_group,
                        c_group_stride, (int)epi, (float)alpha, (int)bn, err.data_ptr<int>(),
                        cur_stream());
  check_rc(rc, "mb_gemm_bf16");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM (dense / grouped)");
}
