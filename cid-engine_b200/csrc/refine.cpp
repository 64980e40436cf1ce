// Host entry of the display refinement policy.  The reference runs the policy
// on host copies of the statistics (csrc/refine.cpp:246-250, 428 of
// fwerkor/cid-engine v1.1.0: four device->host copies and one host->device
// copy per call, i.e. a host sync every decode step); this library validates on
// the host and runs the whole policy on the device (one CTA per row).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "cid_engine/ops.hpp"
#include "cid_engine_b200.h"

namespace cid::engine {

at::Tensor refine_display_from_statistics(
    Backend backend, const at::Tensor& token_ids, const at::Tensor& confidence,
    const at::Tensor& predicted, const at::Tensor& current_confidence,
    std::int64_t mask_token_id, const std::optional<std::int64_t>& eos_token_id,
    double reveal_fraction, double revision_fraction, double revision_margin) {
  TORCH_CHECK(token_ids.dim() == 2, "token_ids must have shape [batch, tokens]");        // :232
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");   // :233
  TORCH_CHECK(predicted.sizes() == token_ids.sizes(), "predicted must match token_ids");  // :234
  TORCH_CHECK(predicted.scalar_type() == at::kLong, "predicted must use torch.int64");   // :235
  TORCH_CHECK(confidence.sizes() == token_ids.sizes(), "confidence must match token_ids");  // :236
  TORCH_CHECK(current_confidence.sizes() == token_ids.sizes(),
              "current_confidence must match token_ids");  // :237-239
  TORCH_CHECK(reveal_fraction >= 0.0 && reveal_fraction <= 1.0,
              "reveal_fraction must be in [0, 1]");  // :240
  TORCH_CHECK(revision_fraction >= 0.0 && revision_fraction <= 1.0,
              "revision_fraction must be in [0, 1]");  // :241-243
  TORCH_CHECK(revision_margin >= 0.0, "revision_margin must be non-negative");  // :244
  auto out = at::empty(token_ids.sizes(), token_ids.options());
  if (backend == Backend::kMeta) return out;
  if (backend == Backend::kCpu) detail::no_cpu_backend("refine_display_from_statistics");
  TORCH_CHECK(confidence.device() == token_ids.device() && predicted.device() == token_ids.device() &&
                  current_confidence.device() == token_ids.device(),
              "cid_engine.refine_display_from_statistics: all tensors must be on the same device");
  if (token_ids.numel() == 0) return out;
  const c10::cuda::CUDAGuard guard(token_ids.device());
  auto ids = token_ids.contiguous();
  auto pred = predicted.contiguous();
  auto conf = confidence.to(at::kFloat).contiguous();  // :249 .to(kFloat)
  auto cur = current_confidence.to(at::kFloat).contiguous();
  auto stream = at::cuda::getCurrentCUDAStream(token_ids.get_device()).stream();
  detail::check_result(
      cid_refine_display(ids.data_ptr<std::int64_t>(), conf.data_ptr<float>(),
                         pred.data_ptr<std::int64_t>(), cur.data_ptr<float>(), ids.size(0),
                         ids.size(1), mask_token_id, eos_token_id.has_value() ? 1 : 0,
                         eos_token_id.value_or(-1), reveal_fraction, revision_fraction,
                         revision_margin, out.data_ptr<std::int64_t>(),
                         reinterpret_cast<void*>(stream)),
      "refine_display_from_statistics");
  return out;
}

}  // namespace cid::engine
