// torch.ops.otq.*: the quantized linear layer registered as PyTorch operators (TORCH_LIBRARY),
// each a thin call into libotq's C ABI (include/otq.h) on the current CUDA stream, with outputs
// allocated by PyTorch's caching allocator (so the ops can be captured in CUDA graphs after a
// first call of each shape). Argument errors the library reports (sizes, alignment, formats)
// raise ValueError, CUDA errors RuntimeError. The reference's operator surface these mirror:
// QACT (opentpu/fp32.py:321-343), MM (opentpu/isasim.py:749-910), QACT + MM as ol.dot emits it
// (opentpu/language.py:150-162), the prefill layer `deq @ x` (opentpu/reference.py:14-17) and
// the greedy sink (opentpu/llm/generate.py:252-280).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "../../include/otq.h"

namespace {

void check(int st, const char* what) {
  if (st == OTQ_OK) return;
  if (st == OTQ_ERR_ARG || st == OTQ_ERR_ALIGN || st == OTQ_ERR_FORMAT)
    TORCH_CHECK_VALUE(false, what, ": ", otq_status_string(st));
  TORCH_CHECK(false, what, ": ", otq_status_string(st), " ", otq_last_cuda_error());
}

void* stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

void need(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK_VALUE(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", wants ", dt);
}

// A 2-D view with unit column stride ([K] becomes [1, K]).
at::Tensor rows2d(const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.dim() == 1 || t.dim() == 2, name, " must be 1-D or 2-D");
  at::Tensor r = t.dim() == 1 ? t.unsqueeze(0) : t;
  if (r.stride(1) != 1) r = r.contiguous();
  return r;
}

const uint8_t* opt_ptr(const c10::optional<at::Tensor>& t, int64_t* stride) {
  if (!t.has_value() || !t->defined()) {
    *stride = 0;
    return nullptr;
  }
  need(*t, at::kByte, "srows");
  TORCH_CHECK_VALUE(t->dim() == 2 && t->stride(1) == 1, "srows must be [N, scale bytes]");
  *stride = t->stride(0);
  return t->data_ptr<uint8_t>();
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> quantize_act(const at::Tensor& x, bool row_mode,
                                                            int64_t group) {
  need(x, at::kFloat, "x");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor x2 = rows2d(x, "x");
  const int64_t M = x2.size(0), K = x2.size(1);
  TORCH_CHECK_VALUE(group > 0 && K % group == 0, "group must divide K");
  auto q = at::empty({M, K}, x.options().dtype(at::kChar));
  auto S = at::empty({M}, x.options());
  auto d = at::empty({M, K / group}, x.options().dtype(at::kByte));
  check(otq_quantize_rows(x2.data_ptr<float>(), M, K, x2.stride(0), static_cast<int>(group),
                          row_mode ? 1 : 0, q.data_ptr<int8_t>(), K, S.data_ptr<float>(),
                          d.data_ptr<uint8_t>(), K / group, stream()),
        "otq.quantize_act");
  return {q, S, d};
}

at::Tensor mm(const at::Tensor& q, const at::Tensor& S, const at::Tensor& d, const at::Tensor& rows,
              const c10::optional<at::Tensor>& srows, int64_t fmt, int64_t flags, int64_t K,
              int64_t k0) {
  need(q, at::kChar, "q");
  need(S, at::kFloat, "S");
  need(d, at::kByte, "d");
  need(rows, at::kByte, "rows");
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK_VALUE(q.dim() == 2 && q.size(1) == K && q.stride(1) == 1, "q must be [M, K]");
  TORCH_CHECK_VALUE(d.dim() == 2 && d.stride(1) == 1 && S.is_contiguous(), "bad S / d");
  TORCH_CHECK_VALUE(rows.dim() == 2 && rows.stride(1) == 1, "rows must be [N, row bytes]");
  const int64_t M = q.size(0), N = rows.size(0);
  int64_t srs = 0;
  const uint8_t* sp = opt_ptr(srows, &srs);
  auto y = at::empty({M, N}, q.options().dtype(at::kFloat));
  check(otq_mm(static_cast<int>(fmt), static_cast<int>(flags), rows.data_ptr<uint8_t>(),
               rows.stride(0), sp, srs, static_cast<int>(k0), N, K, q.data_ptr<int8_t>(),
               q.stride(0), S.data_ptr<float>(), d.data_ptr<uint8_t>(), d.stride(0), M, nullptr,
               y.data_ptr<float>(), N, stream()),
        "otq.mm");
  return y;
}

at::Tensor qlinear(const at::Tensor& x, const at::Tensor& rows,
                   const c10::optional<at::Tensor>& srows, int64_t fmt, int64_t flags, int64_t K,
                   int64_t k0, bool row_mode) {
  need(x, at::kFloat, "x");
  need(rows, at::kByte, "rows");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor x2 = rows2d(x, "x");
  TORCH_CHECK_VALUE(x2.size(1) == K, "x has ", x2.size(1), " columns for K = ", K);
  TORCH_CHECK_VALUE(rows.dim() == 2 && rows.stride(1) == 1, "rows must be [N, row bytes]");
  const int64_t M = x2.size(0), N = rows.size(0);
  int64_t srs = 0;
  const uint8_t* sp = opt_ptr(srows, &srs);
  auto y = at::empty({M, N}, x.options());
  check(otq_qmm(static_cast<int>(fmt), static_cast<int>(flags), rows.data_ptr<uint8_t>(),
                rows.stride(0), sp, srs, static_cast<int>(k0), N, K, x2.data_ptr<float>(),
                x2.stride(0), row_mode ? 1 : 0, M, nullptr, y.data_ptr<float>(), N, stream()),
        "otq.qlinear");
  return x.dim() == 1 ? y.squeeze(0) : y;
}

at::Tensor gemm_w8a16(const at::Tensor& x, const at::Tensor& rows,
                      const c10::optional<at::Tensor>& srows, int64_t flags) {
  need(x, at::kBFloat16, "x");
  need(rows, at::kByte, "rows");
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK_VALUE(x.dim() == 2, "x must be [M, K]");
  at::Tensor xc = (x.stride(1) == 1 && x.stride(0) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0) ? x : x.contiguous();
  TORCH_CHECK_VALUE(rows.dim() == 2 && rows.stride(1) == 1, "rows must be [N, row bytes]");
  const int64_t M = xc.size(0), K = xc.size(1), N = rows.size(0);
  int64_t srs = 0;
  const uint8_t* sp = opt_ptr(srows, &srs);
  auto y = at::empty({M, N}, x.options().dtype(at::kFloat));
  check(otq_gemm_w8a16(static_cast<int>(flags), rows.data_ptr<uint8_t>(), rows.stride(0), sp, srs,
                       N, K, reinterpret_cast<const uint16_t*>(xc.data_ptr()), xc.stride(0), M,
                       y.data_ptr<float>(), N, stream()),
        "otq.gemm_w8a16");
  return y;
}

at::Tensor linear_g32(const at::Tensor& x, const at::Tensor& codes, const at::Tensor& scales) {
  need(x, at::kFloat, "x");
  need(codes, at::kByte, "codes");
  need(scales, at::kHalf, "scales");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor x2 = rows2d(x, "x");
  TORCH_CHECK_VALUE(codes.dim() == 2 && codes.is_contiguous() && scales.is_contiguous(),
                    "codes [N, K/2] and scales [N, K/32] must be contiguous");
  const int64_t M = x2.size(0), K = x2.size(1), N = codes.size(0);
  TORCH_CHECK_VALUE(codes.size(1) * 2 == K && scales.size(0) == N && scales.size(1) * 32 == K,
                    "codes / scales do not fit x's K");
  auto y = at::empty({M, N}, x.options());
  check(otq_linear_g32(codes.data_ptr<uint8_t>(),
                       reinterpret_cast<const uint16_t*>(scales.data_ptr()), N, K,
                       x2.data_ptr<float>(), x2.stride(0), M, 0, y.data_ptr<float>(), N, stream()),
        "otq.linear_g32");
  return x.dim() == 1 ? y.squeeze(0) : y;
}

at::Tensor argmax(const at::Tensor& x) {
  need(x, at::kFloat, "x");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor v = x.dim() == 2 && x.size(0) == 1 ? x.select(0, 0) : x;
  TORCH_CHECK_VALUE(v.dim() == 1, "x must be one row");
  auto out = at::empty({2}, x.options().dtype(at::kLong));
  check(otq_argmax(v.data_ptr<float>(), v.size(0), v.stride(0), out.data_ptr<int64_t>(), stream()),
        "otq.argmax");
  return out.narrow(0, 0, 1);
}

}  // namespace

TORCH_LIBRARY(otq, m) {
  m.def("quantize_act(Tensor x, bool row_mode=False, int group=32) -> (Tensor, Tensor, Tensor)");
  m.def("mm(Tensor q, Tensor S, Tensor d, Tensor rows, Tensor? srows, int fmt, int flags, int K, "
        "int k0=0) -> Tensor");
  m.def("qlinear(Tensor x, Tensor rows, Tensor? srows, int fmt, int flags, int K, int k0=0, "
        "bool row_mode=False) -> Tensor");
  m.def("gemm_w8a16(Tensor x, Tensor rows, Tensor? srows, int flags) -> Tensor");
  m.def("linear_g32(Tensor x, Tensor codes, Tensor scales) -> Tensor");
  m.def("argmax(Tensor x) -> Tensor");
}

TORCH_LIBRARY_IMPL(otq, CUDA, m) {
  m.impl("quantize_act", &quantize_act);
  m.impl("mm", &mm);
  m.impl("qlinear", &qlinear);
  m.impl("gemm_w8a16", &gemm_w8a16);
  m.impl("linear_g32", &linear_g32);
  m.impl("argmax", &argmax);
}
