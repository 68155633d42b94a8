// The torch op exactsample::verify_out, with the reference's schema
// (csrc/bindings.cpp:139-146), as a thin shim over the C ABI: it checks that
// every tensor is on the logits' CUDA device, describes each tensor as an
// es_tensor, and calls es_verify on the current stream. Every other check
// (dtype, rank, shape, capacity, alignment, aliasing) is the C ABI's, and its
// message becomes the RuntimeError.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "exactsample_b200.h"

namespace {
using at::Tensor;
using OptionalTensor = std::optional<Tensor>;

int32_t dtype_of(const Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return ES_F32;
    case at::kDouble: return ES_F64;
    case at::kHalf: return ES_F16;
    case at::kBFloat16: return ES_BF16;
    case at::kInt: return ES_I32;
    case at::kLong: return ES_I64;
    case at::kByte: return ES_U8;
    default: return -1;
  }
}

es_tensor describe(const Tensor& t) {
  es_tensor e{};
  e.data = t.numel() ? const_cast<void*>(t.const_data_ptr()) : nullptr;
  e.dtype = dtype_of(t);
  e.ndim = int32_t(t.dim());
  for (int d = 0; d < t.dim() && d < 2; ++d) {
    e.size[d] = t.size(d);
    e.stride[d] = t.stride(d);
  }
  if (t.dim() > 2 || t.dim() == 0) e.ndim = -1;  // rejected by the C ABI's rank checks (0 would read as absent)
  return e;
}

void verify_out(const Tensor& logits, const Tensor& cu_rows, const Tensor& draft_ids,
                const OptionalTensor& draft_logits, const Tensor& temperature, const Tensor& top_k,
                const Tensor& top_p, const Tensor& min_p, const Tensor& draft_kind, const Tensor& seeds,
                const Tensor& stream_ids, const Tensor& positions, const OptionalTensor& mask, Tensor workspace,
                Tensor tokens, Tensor accepted_len, Tensor status, Tensor path_used, int64_t mode, int64_t dispatch,
                int64_t max_draft, int64_t list_max) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2, "target_logits must be a 2D CUDA tensor");
  const auto device = logits.device();
  auto same_device = [&](const Tensor& t, const char* name) {
    TORCH_CHECK(t.device() == device, name, " has wrong device, dtype or rank");
  };
  same_device(cu_rows, "cu_rows");
  same_device(draft_ids, "draft_ids");
  for (const auto* t : {&temperature, &top_p, &min_p}) same_device(*t, "floating request parameter");
  for (const auto* t : {&top_k, &draft_kind, &seeds, &stream_ids}) same_device(*t, "integer request parameter");
  same_device(positions, "positions");
  if (draft_logits.has_value()) TORCH_CHECK(draft_logits->device() == device, "draft_logits shape/device mismatch");
  if (mask.has_value()) same_device(*mask, "mask");
  same_device(workspace, "workspace");
  same_device(tokens, "tokens");
  for (const auto* t : {&accepted_len, &status, &path_used}) same_device(*t, "output");

  es_args a{};
  a.target_logits = describe(logits);
  a.cu_rows = describe(cu_rows);
  a.draft_ids = describe(draft_ids);
  if (draft_logits.has_value()) a.draft_logits = describe(*draft_logits);
  a.temperature = describe(temperature);
  a.top_k = describe(top_k);
  a.top_p = describe(top_p);
  a.min_p = describe(min_p);
  a.draft_kind = describe(draft_kind);
  a.seeds = describe(seeds);
  a.stream_ids = describe(stream_ids);
  a.positions = describe(positions);
  if (mask.has_value()) a.mask = describe(*mask);
  a.workspace = describe(workspace);
  a.tokens = describe(tokens);
  a.accepted_len = describe(accepted_len);
  a.status = describe(status);
  a.path_used = describe(path_used);
  a.mode = mode;
  a.dispatch = dispatch;
  a.max_draft = max_draft;
  a.list_max = list_max;
  if (a.workspace.ndim == 1 && !workspace.is_contiguous()) a.workspace.stride[0] = 2;  // reported as non-contiguous
  c10::cuda::CUDAGuard guard(device);
  const int result = es_verify(&a, c10::cuda::getCurrentCUDAStream(device.index()).stream());
  TORCH_CHECK(result == ES_SUCCESS, es_last_error());
}
}  // namespace

TORCH_LIBRARY(exactsample, m) {
  m.def(
      "verify_out(Tensor target_logits, Tensor cu_rows, Tensor draft_ids, Tensor? draft_logits, "
      "Tensor temperature, Tensor top_k, Tensor top_p, Tensor min_p, Tensor draft_kind, "
      "Tensor seeds, Tensor stream_ids, Tensor positions, Tensor? mask, "
      "Tensor(a!) workspace, Tensor(b!) tokens, Tensor(c!) accepted_len, Tensor(d!) status, "
      "Tensor(e!) path_used, int mode, int dispatch, int max_draft, int list_max) -> ()");
}
TORCH_LIBRARY_IMPL(exactsample, CUDA, m) { m.impl("verify_out", &verify_out); }
