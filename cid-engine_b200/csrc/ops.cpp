// Host side of the B200 build: validation (with the reference's messages),
// output allocation and C-ABI launches on the current CUDA stream.
//
// Validation follows csrc/ops.cpp of fwerkor/cid-engine v1.1.0 line by line;
// the line of each check is cited.  Nothing here computes on the CPU: with CPU
// tensors every operator validates and then raises (no CPU fallback).
#include "cid_engine/ops.hpp"

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <array>
#include <mutex>
#include <string>

#include "cid_engine_b200.h"

namespace cid::engine {
namespace detail {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return CID_DTYPE_F32;
    case at::kDouble: return CID_DTYPE_F64;
    case at::kHalf: return CID_DTYPE_F16;
    case at::kBFloat16: return CID_DTYPE_BF16;
    case at::kBool: return CID_DTYPE_BOOL;
    case at::kLong: return CID_DTYPE_I64;
    case at::kInt: return CID_DTYPE_I32;
    case at::kByte: return CID_DTYPE_U8;
    case at::kChar: return CID_DTYPE_I8;
    case at::kShort: return CID_DTYPE_I16;
    default: return -1;
  }
}

void check_result(int rc, const char* op) {
  if (rc == CID_OK) return;
  std::string msg = std::string("cid_engine.") + op + ": " + cid_result_string(rc);
  if (rc == CID_ERR_CUDA || rc == CID_ERR_LAUNCH) msg += std::string(" (") + cid_last_cuda_error() + ")";
  TORCH_CHECK(false, msg);
}

namespace {
std::mutex g_status_mutex;
std::array<at::Tensor, 64> g_status;
}  // namespace

std::uint32_t* status_word(const at::Device& device) {
  const auto index = device.index();
  TORCH_CHECK(index >= 0 && index < 64, "cid_engine: device index out of range");
  std::lock_guard<std::mutex> lock(g_status_mutex);
  auto& t = g_status[index];
  if (!t.defined()) t = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(device));
  return reinterpret_cast<std::uint32_t*>(t.data_ptr<int>());
}

[[noreturn]] void no_cpu_backend(const char* op) {
  TORCH_CHECK(false, "cid_engine.", op,
              ": cid-engine-b200 runs on CUDA devices only (sm_100a kernels, no CPU "
              "fallback); move the inputs to a CUDA device");
}

}  // namespace detail

std::int64_t read_device_status(std::int64_t device, bool reset) {
  TORCH_CHECK(device >= 0 && device < 64, "device index out of range");
  const at::Device dev(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  detail::status_word(dev);
  at::Tensor t;
  {
    std::lock_guard<std::mutex> lock(detail::g_status_mutex);
    t = detail::g_status[device];
  }
  const std::int64_t v = static_cast<std::uint32_t>(t.cpu().item<int>());
  if (reset) t.zero_();
  return v;
}

namespace {

using detail::check_result;
using detail::dtype_code;

void* stream_of(const at::Tensor& t) {
  return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

cid_dtype_t dt(const at::Tensor& t) {
  const int c = dtype_code(t.scalar_type());
  TORCH_CHECK(c >= 0, "cid_engine: unsupported dtype ", t.scalar_type());
  return static_cast<cid_dtype_t>(c);
}

void same_device(const char* op, std::initializer_list<const at::Tensor*> ts) {
  const at::Tensor* first = nullptr;
  for (const auto* t : ts) {
    if (!t || !t->defined()) continue;
    if (!first) {
      first = t;
      continue;
    }
    TORCH_CHECK(t->device() == first->device(), "cid_engine.", op,
                ": all tensors must be on the same device");
  }
}

// Rows of a [B, L, V] tensor with unit stride along V and a single row
// stride (b*L + l addressing); otherwise a contiguous copy.
std::pair<at::Tensor, std::int64_t> rows_view(const at::Tensor& logits) {
  const auto B = logits.size(0), L = logits.size(1);
  const bool unit = logits.size(2) <= 1 || logits.stride(2) == 1;
  const auto sl = logits.stride(1), sb = logits.stride(0);
  const bool uniform = B <= 1 || L <= 1 || sb == L * sl;
  if (unit && uniform) {
    std::int64_t rs = L > 1 ? sl : (B > 1 ? sb : logits.size(2));
    if (rs >= logits.size(2) && rs > 0) return {logits, rs};
  }
  auto c = logits.contiguous();
  return {c, c.size(2)};
}

}  // namespace

// ---------------------------------------------------------------------------
// display_token_statistics — csrc/ops.cpp:446-474
// ---------------------------------------------------------------------------

Tensor3 display_token_statistics(Backend backend, const at::Tensor& token_ids,
                                 const at::Tensor& logits) {
  TORCH_CHECK(token_ids.dim() == 2, "token_ids must have shape [batch, tokens]");   // :449
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");  // :450
  TORCH_CHECK(logits.dim() == 3 && logits.size(0) == token_ids.size(0) &&
                  logits.size(1) == token_ids.size(1),
              "logits must have shape [batch, tokens, vocab]");  // :451-455
  TORCH_CHECK(logits.size(-1) > 0, "logits vocabulary dimension must be non-empty");  // :456
  TORCH_CHECK(logits.is_floating_point(), "logits must use a floating dtype");
  same_device("display_token_statistics", {&token_ids, &logits});
  const auto f32 = token_ids.options().dtype(at::kFloat);
  auto confidence = at::empty(token_ids.sizes(), f32);
  auto predicted = at::empty(token_ids.sizes(), token_ids.options().dtype(at::kLong));
  auto current = at::empty(token_ids.sizes(), f32);
  if (backend == Backend::kMeta) return {confidence, predicted, current};
  if (backend == Backend::kCpu) detail::no_cpu_backend("display_token_statistics");
  const std::int64_t rows = token_ids.numel();
  if (rows == 0) return {confidence, predicted, current};
  const c10::cuda::CUDAGuard guard(logits.device());
  auto [lg, row_stride] = rows_view(logits);
  auto ids = token_ids.contiguous();
  check_result(cid_display_token_statistics(
                   dt(lg), lg.data_ptr(), row_stride, ids.data_ptr<std::int64_t>(), rows,
                   lg.size(2), confidence.data_ptr<float>(), predicted.data_ptr<std::int64_t>(),
                   current.data_ptr<float>(), detail::status_word(logits.device()),
                   stream_of(logits)),
               "display_token_statistics");
  return {confidence, predicted, current};
}

// ---------------------------------------------------------------------------
// display_token_statistics_with_repetition — csrc/ops.cpp:477-552
// ---------------------------------------------------------------------------

Tensor3 display_token_statistics_with_repetition(
    Backend backend, const at::Tensor& token_ids, const at::Tensor& logits,
    std::int64_t mask_token_id, const std::optional<std::int64_t>& eos_token_id,
    double repetition_score_multiplier) {
  TORCH_CHECK(repetition_score_multiplier > 0.0 && repetition_score_multiplier <= 1.0,
              "repetition_score_multiplier must be in (0, 1]");  // :484-486
  TORCH_CHECK(token_ids.dim() == 2, "token_ids must have shape [batch, tokens]");  // :487
  TORCH_CHECK(logits.dim() == 3 && logits.size(0) == token_ids.size(0) &&
                  logits.size(1) == token_ids.size(1),
              "logits must have shape [batch, tokens, vocab]");  // :488-492
  if (repetition_score_multiplier == 1.0 || token_ids.size(1) <= 1)  // :494-496
    return display_token_statistics(backend, token_ids, logits);
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");
  TORCH_CHECK(logits.size(-1) > 0, "logits vocabulary dimension must be non-empty");
  TORCH_CHECK(logits.is_floating_point(), "logits must use a floating dtype");
  same_device("display_token_statistics_with_repetition", {&token_ids, &logits});
  const auto f32 = token_ids.options().dtype(at::kFloat);
  auto confidence = at::empty(token_ids.sizes(), f32);
  auto predicted = at::empty(token_ids.sizes(), token_ids.options().dtype(at::kLong));
  auto current = at::empty(token_ids.sizes(), f32);
  if (backend == Backend::kMeta) return {confidence, predicted, current};
  if (backend == Backend::kCpu) detail::no_cpu_backend("display_token_statistics_with_repetition");
  if (token_ids.numel() == 0) return {confidence, predicted, current};
  const c10::cuda::CUDAGuard guard(logits.device());
  auto [lg, row_stride] = rows_view(logits);
  auto ids = token_ids.contiguous();
  check_result(cid_display_token_statistics_with_repetition(
                   dt(lg), lg.data_ptr(), row_stride, ids.data_ptr<std::int64_t>(),
                   ids.size(0), ids.size(1), lg.size(2), mask_token_id,
                   eos_token_id.has_value() ? 1 : 0, eos_token_id.value_or(-1),
                   repetition_score_multiplier, confidence.data_ptr<float>(),
                   predicted.data_ptr<std::int64_t>(), current.data_ptr<float>(),
                   detail::status_word(logits.device()), stream_of(logits)),
               "display_token_statistics_with_repetition");
  return {confidence, predicted, current};
}

// ---------------------------------------------------------------------------
// Vocabulary-parallel statistics (additive to the reference's operators)
// ---------------------------------------------------------------------------

at::Tensor display_shard_records(Backend backend, const at::Tensor& token_ids,
                                 const at::Tensor& logits_shard, std::int64_t vocab_offset,
                                 std::int64_t total_vocab) {
  TORCH_CHECK(token_ids.dim() == 2, "token_ids must have shape [batch, tokens]");
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");
  TORCH_CHECK(logits_shard.dim() == 3 && logits_shard.size(0) == token_ids.size(0) &&
                  logits_shard.size(1) == token_ids.size(1),
              "logits must have shape [batch, tokens, vocab]");
  TORCH_CHECK(logits_shard.size(-1) > 0, "logits vocabulary dimension must be non-empty");
  TORCH_CHECK(vocab_offset >= 0 && vocab_offset + logits_shard.size(-1) <= total_vocab,
              "vocabulary shard must lie inside [0, total_vocab)");
  same_device("display_shard_records", {&token_ids, &logits_shard});
  // one 16-byte record per row, stored as 4 x int32
  auto records = at::empty({token_ids.numel(), 4}, token_ids.options().dtype(at::kInt));
  if (backend == Backend::kMeta) return records;
  if (backend == Backend::kCpu) detail::no_cpu_backend("display_shard_records");
  if (token_ids.numel() == 0) return records;
  const c10::cuda::CUDAGuard guard(logits_shard.device());
  auto [lg, row_stride] = rows_view(logits_shard);
  auto ids = token_ids.contiguous();
  check_result(cid_display_shard_records(
                   dt(lg), lg.data_ptr(), row_stride, ids.data_ptr<std::int64_t>(), ids.numel(),
                   lg.size(2), vocab_offset, total_vocab,
                   reinterpret_cast<cid_shard_record_t*>(records.data_ptr<int>()),
                   detail::status_word(lg.device()), stream_of(lg)),
               "display_shard_records");
  return records;
}

Tensor3 display_combine_records(Backend backend, const at::Tensor& records,
                                const at::Tensor& token_ids, at::IntArrayRef shard_offsets) {
  const auto world = static_cast<std::int64_t>(shard_offsets.size()) - 1;
  TORCH_CHECK(world >= 1, "shard_offsets must hold world_size + 1 offsets");
  TORCH_CHECK(token_ids.dim() == 2 && token_ids.scalar_type() == at::kLong,
              "token_ids must be an int64 [batch, tokens] tensor");
  TORCH_CHECK(records.scalar_type() == at::kInt && records.dim() == 3 &&
                  records.size(0) == world && records.size(1) == token_ids.numel() &&
                  records.size(2) == 4,
              "records must be int32 [world, rows, 4]");
  same_device("display_combine_records", {&records, &token_ids});
  const auto f32 = token_ids.options().dtype(at::kFloat);
  auto confidence = at::empty(token_ids.sizes(), f32);
  auto predicted = at::empty(token_ids.sizes(), token_ids.options().dtype(at::kLong));
  auto current = at::empty(token_ids.sizes(), f32);
  if (backend == Backend::kMeta) return {confidence, predicted, current};
  if (backend == Backend::kCpu) detail::no_cpu_backend("display_combine_records");
  if (token_ids.numel() == 0) return {confidence, predicted, current};
  const c10::cuda::CUDAGuard guard(records.device());
  auto rec = records.contiguous();
  auto ids = token_ids.contiguous();
  std::vector<std::int64_t> offs(shard_offsets.begin(), shard_offsets.end());
  check_result(cid_display_combine_records(
                   reinterpret_cast<const cid_shard_record_t*>(rec.data_ptr<int>()),
                   static_cast<int>(world), offs.data(), ids.data_ptr<std::int64_t>(),
                   ids.numel(), confidence.data_ptr<float>(), predicted.data_ptr<std::int64_t>(),
                   current.data_ptr<float>(), detail::status_word(rec.device()), stream_of(rec)),
               "display_combine_records");
  return {confidence, predicted, current};
}

Tensor3 lm_head_display_statistics(Backend backend, const at::Tensor& token_ids,
                                   const at::Tensor& hidden, const at::Tensor& weight,
                                   bool round_bf16) {
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");
  TORCH_CHECK(hidden.dim() >= 1 && hidden.dim() - 1 == token_ids.dim() &&
                  hidden.sizes().slice(0, hidden.dim() - 1) == token_ids.sizes(),
              "hidden must have shape [*token_ids.shape, hidden_dim]");
  TORCH_CHECK(weight.dim() == 2 && weight.size(1) == hidden.size(-1),
              "weight must have shape [vocab, hidden_dim]");
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16,
              "hidden and weight must use torch.bfloat16");
  TORCH_CHECK(weight.size(0) > 0, "weight vocabulary dimension must be non-empty");
  TORCH_CHECK(hidden.size(-1) % 8 == 0, "hidden_dim must be a multiple of 8");
  same_device("lm_head_display_statistics", {&token_ids, &hidden, &weight});
  const auto f32 = token_ids.options().dtype(at::kFloat);
  auto confidence = at::empty(token_ids.sizes(), f32);
  auto predicted = at::empty(token_ids.sizes(), token_ids.options().dtype(at::kLong));
  auto current = at::empty(token_ids.sizes(), f32);
  if (backend == Backend::kMeta) return {confidence, predicted, current};
  if (backend == Backend::kCpu) detail::no_cpu_backend("lm_head_display_statistics");
  if (token_ids.numel() == 0) return {confidence, predicted, current};
  const c10::cuda::CUDAGuard guard(hidden.device());
  auto h = hidden.contiguous();
  auto w = weight.contiguous();
  auto ids = token_ids.contiguous();
  const auto rows = ids.numel();
  const size_t ws_bytes = cid_lm_head_workspace_bytes(rows, w.size(0));
  auto workspace = at::empty({static_cast<std::int64_t>(ws_bytes)},
                             hidden.options().dtype(at::kByte));
  check_result(cid_lm_head_display_statistics(
                   h.data_ptr(), rows, h.size(-1), w.data_ptr(), w.size(0),
                   ids.data_ptr<std::int64_t>(), round_bf16 ? 1 : 0,
                   confidence.data_ptr<float>(), predicted.data_ptr<std::int64_t>(),
                   current.data_ptr<float>(), workspace.data_ptr(), ws_bytes,
                   detail::status_word(h.device()), stream_of(h)),
               "lm_head_display_statistics");
  return {confidence, predicted, current};
}

at::Tensor lm_head_shard_records(Backend backend, const at::Tensor& token_ids,
                                 const at::Tensor& hidden, const at::Tensor& weight_shard,
                                 std::int64_t vocab_offset, std::int64_t total_vocab,
                                 bool round_bf16) {
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");
  TORCH_CHECK(hidden.dim() >= 1 && hidden.dim() - 1 == token_ids.dim() &&
                  hidden.sizes().slice(0, hidden.dim() - 1) == token_ids.sizes(),
              "hidden must have shape [*token_ids.shape, hidden_dim]");
  TORCH_CHECK(weight_shard.dim() == 2 && weight_shard.size(1) == hidden.size(-1),
              "weight must have shape [vocab, hidden_dim]");
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && weight_shard.scalar_type() == at::kBFloat16,
              "hidden and weight must use torch.bfloat16");
  TORCH_CHECK(weight_shard.size(0) > 0, "weight vocabulary dimension must be non-empty");
  TORCH_CHECK(hidden.size(-1) % 8 == 0, "hidden_dim must be a multiple of 8");
  TORCH_CHECK(vocab_offset >= 0 && vocab_offset + weight_shard.size(0) <= total_vocab,
              "vocabulary shard must lie inside [0, total_vocab)");
  same_device("lm_head_shard_records", {&token_ids, &hidden, &weight_shard});
  auto records = at::empty({token_ids.numel(), 4}, token_ids.options().dtype(at::kInt));
  if (backend == Backend::kMeta) return records;
  if (backend == Backend::kCpu) detail::no_cpu_backend("lm_head_shard_records");
  if (token_ids.numel() == 0) return records;
  const c10::cuda::CUDAGuard guard(hidden.device());
  auto h = hidden.contiguous();
  auto w = weight_shard.contiguous();
  auto ids = token_ids.contiguous();
  const auto rows = ids.numel();
  const size_t ws_bytes = cid_lm_head_workspace_bytes(rows, w.size(0));
  auto workspace = at::empty({static_cast<std::int64_t>(ws_bytes)},
                             hidden.options().dtype(at::kByte));
  check_result(cid_lm_head_shard_records(
                   h.data_ptr(), rows, h.size(-1), w.data_ptr(), w.size(0), vocab_offset,
                   total_vocab, ids.data_ptr<std::int64_t>(), round_bf16 ? 1 : 0,
                   reinterpret_cast<cid_shard_record_t*>(records.data_ptr<int>()),
                   workspace.data_ptr(), ws_bytes, detail::status_word(h.device()),
                   stream_of(h)),
               "lm_head_shard_records");
  return records;
}

// ---------------------------------------------------------------------------
// live_slot_occupancy — csrc/ops.cpp:12-39
// ---------------------------------------------------------------------------

at::Tensor live_slot_occupancy(Backend backend, const at::Tensor& slot_occupancy,
                               const std::optional<at::Tensor>& lifecycle_features,
                               std::int64_t retired_index) {
  TORCH_CHECK(slot_occupancy.dim() == 3 && slot_occupancy.size(-1) == 1,
              "slot_occupancy must have shape [batch, slots, 1]");  // :16-18
  at::ScalarType out_t = slot_occupancy.is_floating_point() ? slot_occupancy.scalar_type()
                                                              : at::kFloat;
  const at::Tensor* life = nullptr;
  if (lifecycle_features.has_value() && lifecycle_features->defined()) {
    life = &*lifecycle_features;
    TORCH_CHECK(life->dim() == 3 && life->size(0) == slot_occupancy.size(0) &&
                    life->size(1) == slot_occupancy.size(1),
                "lifecycle_features must match batch and slot dimensions");  // :26-30
    TORCH_CHECK(retired_index >= 0 && retired_index < life->size(-1),
                "retired_index is outside lifecycle_features");  // :31-33
    const auto lt = life->is_floating_point() ? life->scalar_type() : at::kFloat;
    out_t = at::promote_types(out_t, lt);
    same_device("live_slot_occupancy", {&slot_occupancy, life});
  }
  auto out = at::empty(slot_occupancy.sizes(), slot_occupancy.options().dtype(out_t));
  if (backend == Backend::kMeta) return out;
  if (backend == Backend::kCpu) detail::no_cpu_backend("live_slot_occupancy");
  if (out.numel() == 0) return out;
  const c10::cuda::CUDAGuard guard(slot_occupancy.device());
  auto occ = slot_occupancy.to(out_t).contiguous();
  at::Tensor lc;
  if (life) lc = life->to(out_t).contiguous();
  check_result(cid_live_slot_occupancy(dt(out), occ.data_ptr(), life ? lc.data_ptr() : nullptr,
                                       occ.numel(), life ? lc.size(-1) : 0, retired_index,
                                       out.data_ptr(), stream_of(occ)),
               "live_slot_occupancy");
  return out;
}

// ---------------------------------------------------------------------------
// prefix_allocation_mask — csrc/ops.cpp:41-65
// ---------------------------------------------------------------------------

at::Tensor prefix_allocation_mask(Backend backend, const at::Tensor& occupancy_input,
                                  const at::Tensor& allocation_logits, double threshold,
                                  std::int64_t max_allocations) {
  TORCH_CHECK(occupancy_input.dim() == 2 ||
                  (occupancy_input.dim() == 3 && occupancy_input.size(-1) == 1),
              "occupancy must have shape [batch, slots] or [batch, slots, 1]");  // :46-49
  TORCH_CHECK(threshold >= 0.0 && threshold <= 1.0, "threshold must be in [0, 1]");  // :50
  TORCH_CHECK(max_allocations > 0, "max_allocations must be positive");              // :51
  auto occupancy = occupancy_input.dim() == 3 ? occupancy_input.squeeze(-1) : occupancy_input;
  TORCH_CHECK(allocation_logits.dim() == 2 && allocation_logits.sizes() == occupancy.sizes(),
              "occupancy and allocation_logits must have matching shapes");  // :54-56
  same_device("prefix_allocation_mask", {&occupancy_input, &allocation_logits});
  auto out = at::empty(occupancy.sizes(), occupancy.options().dtype(at::kBool));
  if (backend == Backend::kMeta) return out;
  if (backend == Backend::kCpu) detail::no_cpu_backend("prefix_allocation_mask");
  if (out.numel() == 0) return out;
  const c10::cuda::CUDAGuard guard(occupancy.device());
  at::Tensor lg = allocation_logits;
  if (!lg.is_floating_point()) lg = lg.to(at::kFloat);  // :59 .to(kFloat)
  at::Tensor occ = occupancy;
  if (dtype_code(occ.scalar_type()) < 0) occ = occ.to(at::kBool);
  check_result(cid_prefix_allocation_mask(dt(occ), occ.data_ptr(), occ.stride(0), occ.stride(1),
                                          dt(lg), lg.data_ptr(), lg.stride(0), lg.stride(1),
                                          occ.size(0), occ.size(1), threshold, max_allocations,
                                          reinterpret_cast<std::uint8_t*>(out.data_ptr<bool>()),
                                          stream_of(occ)),
               "prefix_allocation_mask");
  return out;
}

// ---------------------------------------------------------------------------
// batched_linear_assignment — csrc/ops.cpp:68-175
// ---------------------------------------------------------------------------

at::Tensor batched_linear_assignment(Backend backend, const at::Tensor& costs,
                                     const at::Tensor& row_counts) {
  TORCH_CHECK(costs.dim() == 3, "costs must have shape [batch, rows, columns]");  // :71
  TORCH_CHECK(costs.is_floating_point(), "costs must use a floating dtype");        // :72
  TORCH_CHECK(costs.size(1) <= costs.size(2), "assignment rows cannot exceed columns");
  TORCH_CHECK(costs.size(2) <= 16, "batched_linear_assignment supports at most 16 columns");
  TORCH_CHECK(row_counts.dim() == 1 && row_counts.size(0) == costs.size(0),
              "row_counts must have shape [batch]");
  TORCH_CHECK(row_counts.scalar_type() == at::kLong, "row_counts must use torch.int64");
  same_device("batched_linear_assignment", {&costs, &row_counts});
  auto out = at::empty({costs.size(0), costs.size(1)}, costs.options().dtype(at::kLong));
  if (backend == Backend::kMeta) return out;
  if (backend == Backend::kCpu) detail::no_cpu_backend("batched_linear_assignment");
  if (out.numel() == 0) return out;
  const c10::cuda::CUDAGuard guard(costs.device());
  auto c = costs.contiguous();
  auto counts = row_counts.contiguous();
  check_result(cid_batched_linear_assignment(dt(c), c.data_ptr(), counts.data_ptr<std::int64_t>(),
                                             c.size(0), c.size(1), c.size(2),
                                             out.data_ptr<std::int64_t>(),
                                             detail::status_word(c.device()), stream_of(c)),
               "batched_linear_assignment");
  return out;
}

// ---------------------------------------------------------------------------
// rollout_slot_transition — csrc/ops.cpp:184-256
// ---------------------------------------------------------------------------

namespace {

// rollout_slot_transition; with `live_out` also the live occupancy of the
// next state (one kernel, cid_rollout_slot_transition_live).
Tensor6 rollout_common(Backend backend, const at::Tensor& occupancy_input,
                       const at::Tensor& allocation_logits, const at::Tensor& lifecycle_logits,
                       const at::Tensor& revision_logits, const at::Tensor& input_lifecycle,
                       double threshold, std::int64_t max_allocations,
                       std::int64_t retired_index, at::Tensor* live_out) {
  TORCH_CHECK(occupancy_input.dim() == 2 ||
                  (occupancy_input.dim() == 3 && occupancy_input.size(-1) == 1),
              "occupancy must have shape [batch, slots] or [batch, slots, 1]");  // :193-196
  auto occupancy = occupancy_input.dim() == 3 ? occupancy_input.squeeze(-1) : occupancy_input;
  const auto batch = occupancy.size(0);
  const auto slots = occupancy.size(1);
  TORCH_CHECK(allocation_logits.sizes() == occupancy.sizes(),
              "allocation_logits must match occupancy shape");  // :201-203
  TORCH_CHECK(lifecycle_logits.dim() == 3 && lifecycle_logits.size(0) == batch &&
                  lifecycle_logits.size(1) == slots,
              "lifecycle_logits must have shape [batch, slots, lifecycles]");  // :204-208
  TORCH_CHECK(revision_logits.dim() == 3 && revision_logits.size(0) == batch &&
                  revision_logits.size(1) == slots,
              "revision_logits must have shape [batch, slots, revisions]");  // :209-213
  TORCH_CHECK(input_lifecycle.dim() == 3 && input_lifecycle.size(0) == batch &&
                  input_lifecycle.size(1) == slots,
              "input_lifecycle must have shape [batch, slots, lifecycles]");  // :214-218
  TORCH_CHECK(lifecycle_logits.size(-1) == input_lifecycle.size(-1),
              "predicted and input lifecycle widths must match");  // :219-221
  TORCH_CHECK(retired_index >= 0 && retired_index < lifecycle_logits.size(-1),
              "retired_index is outside lifecycle width");  // :222-224
  TORCH_CHECK(threshold >= 0.0 && threshold <= 1.0, "threshold must be in [0, 1]");  // :225
  TORCH_CHECK(max_allocations > 0, "max_allocations must be positive");              // :226
  TORCH_CHECK(revision_logits.size(-1) > 0, "revision_logits must be non-empty");
  same_device("rollout_slot_transition", {&occupancy_input, &allocation_logits,
                                          &lifecycle_logits, &revision_logits,
                                          &input_lifecycle});
  const auto o = occupancy.options();
  auto next = at::empty({batch, slots}, o.dtype(at::kBool));
  auto li = at::empty({batch, slots}, o.dtype(at::kLong));
  auto ri = at::empty({batch, slots}, o.dtype(at::kLong));
  auto ii = at::empty({batch, slots}, o.dtype(at::kLong));
  auto present = at::empty({batch, slots}, o.dtype(at::kBool));
  auto live = at::empty({batch, slots}, o.dtype(at::kBool));
  if (live_out) {
    TORCH_CHECK(lifecycle_logits.is_floating_point(), "lifecycle_logits must use a floating dtype");
    *live_out = at::empty({batch, slots, 1}, lifecycle_logits.options());
  }
  if (backend == Backend::kMeta) return {next, li, ri, ii, present, live};
  if (backend == Backend::kCpu) detail::no_cpu_backend("rollout_slot_transition");
  if (batch == 0 || slots == 0) return {next, li, ri, ii, present, live};
  const c10::cuda::CUDAGuard guard(occupancy.device());
  // one element type for the four float inputs: their promotion (exact, so
  // argmax comparisons are unchanged)
  auto common = at::promote_types(
      at::promote_types(allocation_logits.scalar_type(), lifecycle_logits.scalar_type()),
      at::promote_types(revision_logits.scalar_type(), input_lifecycle.scalar_type()));
  if (!at::isFloatingType(common)) common = at::kFloat;
  auto al = allocation_logits.to(common).contiguous();
  auto lc = lifecycle_logits.to(common).contiguous();
  auto rv = revision_logits.to(common).contiguous();
  auto il = input_lifecycle.to(common).contiguous();
  at::Tensor occ = occupancy.contiguous();
  if (dtype_code(occ.scalar_type()) < 0) occ = occ.to(at::kBool);
  auto u8 = [](at::Tensor& t) { return reinterpret_cast<std::uint8_t*>(t.data_ptr<bool>()); };
  if (live_out) {
    check_result(cid_rollout_slot_transition_live(
                     dt(occ), occ.data_ptr(), dt(al), al.data_ptr(), lc.data_ptr(),
                     rv.data_ptr(), il.data_ptr(), batch, slots, lc.size(-1), rv.size(-1),
                     threshold, max_allocations, retired_index, u8(next),
                     li.data_ptr<std::int64_t>(), ri.data_ptr<std::int64_t>(),
                     ii.data_ptr<std::int64_t>(), u8(present), u8(live), dt(*live_out),
                     live_out->data_ptr(), stream_of(occ)),
                 "rollout_slot_transition_with_live");
    return {next, li, ri, ii, present, live};
  }
  check_result(cid_rollout_slot_transition(
                   dt(occ), occ.data_ptr(), dt(al), al.data_ptr(), lc.data_ptr(), rv.data_ptr(),
                   il.data_ptr(), batch, slots, lc.size(-1), rv.size(-1), threshold,
                   max_allocations, retired_index, u8(next), li.data_ptr<std::int64_t>(),
                   ri.data_ptr<std::int64_t>(), ii.data_ptr<std::int64_t>(), u8(present),
                   u8(live), stream_of(occ)),
               "rollout_slot_transition");
  return {next, li, ri, ii, present, live};
}

}  // namespace

Tensor6 rollout_slot_transition(Backend backend, const at::Tensor& occupancy,
                                const at::Tensor& allocation_logits,
                                const at::Tensor& lifecycle_logits,
                                const at::Tensor& revision_logits,
                                const at::Tensor& input_lifecycle, double threshold,
                                std::int64_t max_allocations, std::int64_t retired_index) {
  return rollout_common(backend, occupancy, allocation_logits, lifecycle_logits, revision_logits,
                        input_lifecycle, threshold, max_allocations, retired_index, nullptr);
}

// Additive: the decode step's rollout and the live occupancy of its next
// state (live_slot_occupancy(next.unsqueeze(-1).to(lifecycle dtype),
// lifecycle_logits, retired_index)) from one kernel.
Tensor7 rollout_slot_transition_with_live(Backend backend, const at::Tensor& occupancy,
                                          const at::Tensor& allocation_logits,
                                          const at::Tensor& lifecycle_logits,
                                          const at::Tensor& revision_logits,
                                          const at::Tensor& input_lifecycle, double threshold,
                                          std::int64_t max_allocations,
                                          std::int64_t retired_index) {
  at::Tensor live_occ;
  auto r = rollout_common(backend, occupancy, allocation_logits, lifecycle_logits,
                          revision_logits, input_lifecycle, threshold, max_allocations,
                          retired_index, &live_occ);
  return {std::get<0>(r), std::get<1>(r), std::get<2>(r), std::get<3>(r), std::get<4>(r),
          std::get<5>(r), live_occ};
}

// ---------------------------------------------------------------------------
// thought_corrupt_from_epsilon — csrc/ops.cpp:258-290
// ---------------------------------------------------------------------------

Tensor3 thought_corrupt_from_epsilon(Backend backend, const at::Tensor& semantic,
                                     const at::Tensor& timesteps, const at::Tensor& occupancy,
                                     const at::Tensor& epsilon) {
  TORCH_CHECK(semantic.dim() == 3, "semantic must have shape [batch, slots, hidden]");  // :263
  TORCH_CHECK(timesteps.dim() == 2 && timesteps.size(0) == semantic.size(0) &&
                  timesteps.size(1) == semantic.size(1),
              "timesteps must have shape [batch, slots]");  // :264-268
  TORCH_CHECK(occupancy.dim() == 3 && occupancy.size(0) == semantic.size(0) &&
                  occupancy.size(1) == semantic.size(1) && occupancy.size(2) == 1,
              "occupancy must have shape [batch, slots, 1]");  // :269-274
  TORCH_CHECK(epsilon.sizes() == semantic.sizes(), "epsilon must match semantic");  // :275
  TORCH_CHECK(semantic.is_floating_point() && timesteps.is_floating_point(),
              "semantic and timesteps must use floating dtypes");
  TORCH_CHECK(epsilon.scalar_type() == semantic.scalar_type(),
              "epsilon must share semantic dtype");
  same_device("thought_corrupt_from_epsilon", {&semantic, &timesteps, &occupancy, &epsilon});
  auto corrupted = at::empty(semantic.sizes(), semantic.options());
  auto local = at::empty({semantic.size(0), semantic.size(1), 1}, semantic.options());
  auto masked = at::empty(semantic.sizes(), semantic.options());
  if (backend == Backend::kMeta) return {corrupted, local, masked};
  if (backend == Backend::kCpu) detail::no_cpu_backend("thought_corrupt_from_epsilon");
  const auto rows = semantic.size(0) * semantic.size(1);
  if (rows == 0) return {corrupted, local, masked};
  const c10::cuda::CUDAGuard guard(semantic.device());
  auto sem = semantic.contiguous();
  auto ts = timesteps.contiguous();
  auto occ = occupancy.contiguous();
  if (dtype_code(occ.scalar_type()) < 0) occ = occ.to(at::kBool);
  auto eps = epsilon.contiguous();
  check_result(cid_thought_corrupt(dt(sem), sem.data_ptr(), dt(ts), ts.data_ptr(), dt(occ),
                                   occ.data_ptr(), eps.data_ptr(), rows, sem.size(2),
                                   corrupted.data_ptr(), local.data_ptr(), masked.data_ptr(),
                                   stream_of(sem)),
               "thought_corrupt_from_epsilon");
  return {corrupted, local, masked};
}

// ---------------------------------------------------------------------------
// display_corrupt_from_random — csrc/ops.cpp:292-391
// ---------------------------------------------------------------------------

Tensor4 display_corrupt_from_random(Backend backend, const at::Tensor& token_ids,
                                    const at::Tensor& timesteps, const at::Tensor& eligible_mask,
                                    const at::Tensor& corruption_random,
                                    const std::optional<at::Tensor>& replacement_random,
                                    const std::optional<at::Tensor>& replacement_offsets,
                                    std::int64_t mask_token_id,
                                    const std::optional<std::int64_t>& eos_token_id,
                                    std::int64_t vocab_size, double replacement_fraction) {
  TORCH_CHECK(token_ids.dim() == 2, "token_ids must have shape [batch, tokens]");       // :304
  TORCH_CHECK(token_ids.scalar_type() == at::kLong, "token_ids must use torch.int64");  // :305
  const auto batch = token_ids.size(0);
  TORCH_CHECK(timesteps.dim() == 1 && timesteps.size(0) == batch,
              "timesteps must have shape [batch]");  // :308-310
  TORCH_CHECK(eligible_mask.sizes() == token_ids.sizes(),
              "eligible_mask must match token_ids shape");  // :311-313
  TORCH_CHECK(corruption_random.sizes() == token_ids.sizes(),
              "corruption_random must match token_ids shape");  // :314-316
  TORCH_CHECK(timesteps.is_floating_point() && corruption_random.is_floating_point(),
              "timesteps and corruption_random must use floating dtypes");  // :317-319
  TORCH_CHECK(replacement_fraction >= 0.0 && replacement_fraction <= 1.0,
              "replacement_fraction must be in [0, 1]");  // :320-322
  const bool replace = replacement_fraction > 0.0;
  const at::Tensor* rr = nullptr;
  const at::Tensor* ro = nullptr;
  if (replace) {  // :343-360
    TORCH_CHECK(vocab_size >= 3, "visible replacement corruption requires vocab_size >= 3");
    TORCH_CHECK(replacement_random.has_value() && replacement_offsets.has_value(),
                "replacement random tensors are required when replacement_fraction > 0");
    rr = &*replacement_random;
    ro = &*replacement_offsets;
    TORCH_CHECK(rr->sizes() == token_ids.sizes(), "replacement_random must match token_ids shape");
    TORCH_CHECK(ro->sizes() == token_ids.sizes(), "replacement_offsets must match token_ids shape");
    TORCH_CHECK(rr->is_floating_point(), "replacement_random must use a floating dtype");
    TORCH_CHECK(ro->scalar_type() == at::kLong, "replacement_offsets must use torch.int64");
  }
  same_device("display_corrupt_from_random",
              {&token_ids, &timesteps, &eligible_mask, &corruption_random, rr, ro});
  auto corrupted = at::empty(token_ids.sizes(), token_ids.options());
  auto labels = at::empty(token_ids.sizes(), token_ids.options());
  auto masked = at::empty(token_ids.sizes(), token_ids.options().dtype(at::kBool));
  auto replaced = at::empty(token_ids.sizes(), token_ids.options().dtype(at::kBool));
  if (backend == Backend::kMeta) return {corrupted, labels, masked, replaced};
  if (backend == Backend::kCpu) detail::no_cpu_backend("display_corrupt_from_random");
  if (token_ids.numel() == 0) return {corrupted, labels, masked, replaced};
  const c10::cuda::CUDAGuard guard(token_ids.device());
  auto ids = token_ids.contiguous();
  auto ts = timesteps.contiguous();
  auto el = eligible_mask.contiguous();
  if (dtype_code(el.scalar_type()) < 0) el = el.to(at::kBool);
  auto cr = corruption_random.contiguous();
  at::Tensor rrc, roc;
  if (replace) {
    rrc = rr->contiguous();
    roc = ro->contiguous();
  }
  auto u8 = [](at::Tensor& t) { return reinterpret_cast<std::uint8_t*>(t.data_ptr<bool>()); };
  check_result(cid_display_corrupt(
                   ids.data_ptr<std::int64_t>(), dt(ts), ts.data_ptr(), dt(el), el.data_ptr(),
                   dt(cr), cr.data_ptr(), replace ? dt(rrc) : CID_DTYPE_F32,
                   replace ? rrc.data_ptr() : nullptr,
                   replace ? roc.data_ptr<std::int64_t>() : nullptr, batch, ids.size(1),
                   mask_token_id, eos_token_id.has_value() ? 1 : 0, eos_token_id.value_or(-1),
                   vocab_size, replacement_fraction, corrupted.data_ptr<std::int64_t>(),
                   labels.data_ptr<std::int64_t>(), u8(masked), u8(replaced), stream_of(ids)),
               "display_corrupt_from_random");
  return {corrupted, labels, masked, replaced};
}

// ---------------------------------------------------------------------------
// masked_diffusion_corrupt_from_random — csrc/ops.cpp:394-444
// ---------------------------------------------------------------------------


Tensor4 masked_diffusion_corrupt_from_random(Backend backend, const at::Tensor& clean_ids,
                                             const at::Tensor& ratio_random,
                                             const at::Tensor& mask_random,
                                             std::int64_t mask_token_id, double min_mask_ratio,
                                             double max_mask_ratio) {
  TORCH_CHECK(clean_ids.dim() == 2, "clean_ids must have shape [batch, tokens]");       // :402
  TORCH_CHECK(clean_ids.scalar_type() == at::kLong, "clean_ids must use torch.int64");  // :403
  const auto batch = clean_ids.size(0);
  const auto tokens = clean_ids.size(1);
  TORCH_CHECK(batch > 0 && tokens > 0, "clean_ids dimensions must be non-empty");  // :406
  TORCH_CHECK(ratio_random.sizes() == at::IntArrayRef({batch, 1}),
              "ratio_random must have shape [batch, 1]");  // :407-409
  TORCH_CHECK(mask_random.sizes() == clean_ids.sizes(),
              "mask_random must match clean_ids shape");  // :410-412
  TORCH_CHECK(ratio_random.is_floating_point() && mask_random.is_floating_point(),
              "random tensors must use floating dtypes");  // :413-415
  TORCH_CHECK(min_mask_ratio > 0.0 && min_mask_ratio <= max_mask_ratio && max_mask_ratio <= 1.0,
              "mask ratio range must satisfy 0 < min <= max <= 1");  // :416-420
  same_device("masked_diffusion_corrupt_from_random", {&clean_ids, &ratio_random, &mask_random});
  auto corrupted = at::empty(clean_ids.sizes(), clean_ids.options());
  auto masked = at::empty(clean_ids.sizes(), clean_ids.options().dtype(at::kBool));
  auto ratio = at::empty({batch, 1}, clean_ids.options().dtype(at::kFloat));
  auto metrics = at::empty({2}, clean_ids.options().dtype(at::kFloat));
  if (backend == Backend::kMeta) return {corrupted, masked, ratio, metrics};
  if (backend == Backend::kCpu) detail::no_cpu_backend("masked_diffusion_corrupt_from_random");
  const c10::cuda::CUDAGuard guard(clean_ids.device());
  auto clean = clean_ids.contiguous();
  auto rr = ratio_random.to(at::kFloat).contiguous();  // :422
  auto mr = mask_random.to(at::kFloat).contiguous();   // :423
  const auto ws_bytes = static_cast<std::int64_t>(cid_masked_diffusion_workspace_bytes(batch));
  auto ws = at::empty({(ws_bytes + 7) / 8}, clean_ids.options().dtype(at::kLong));
  check_result(cid_masked_diffusion_corrupt(
                   clean.data_ptr<std::int64_t>(), rr.data_ptr<float>(), mr.data_ptr<float>(),
                   batch, tokens, mask_token_id, min_mask_ratio, max_mask_ratio,
                   corrupted.data_ptr<std::int64_t>(),
                   reinterpret_cast<std::uint8_t*>(masked.data_ptr<bool>()),
                   ratio.data_ptr<float>(), metrics.data_ptr<float>(), ws.data_ptr(),
                   stream_of(clean)),
               "masked_diffusion_corrupt_from_random");
  return {corrupted, masked, ratio, metrics};
}

// ---------------------------------------------------------------------------
// materialize_cell_snapshot — csrc/ops.cpp:556-615
// ---------------------------------------------------------------------------

at::Tensor materialize_cell_snapshot(Backend backend, const at::Tensor& thought_semantic,
                                     const at::Tensor& role_logits,
                                     const at::Tensor& uncertainty,
                                     const at::Tensor& noise_delta,
                                     const at::Tensor& lifecycle_logits,
                                     const at::Tensor& selected,
                                     const at::Tensor& semantic_indices) {
  TORCH_CHECK(thought_semantic.dim() == 3,
              "thought_semantic must have shape [batch, slots, hidden]");  // :564-566
  const auto batch = thought_semantic.size(0);
  const auto slots = thought_semantic.size(1);
  const auto hidden = thought_semantic.size(2);
  TORCH_CHECK(role_logits.dim() == 3 && role_logits.size(0) == batch &&
                  role_logits.size(1) == slots,
              "role_logits must have shape [batch, slots, roles]");  // :570-574
  TORCH_CHECK(uncertainty.sizes() == at::IntArrayRef({batch, slots, 1}),
              "uncertainty must have shape [batch, slots, 1]");  // :575-577
  TORCH_CHECK(noise_delta.sizes() == at::IntArrayRef({batch, slots, 1}),
              "noise_delta must have shape [batch, slots, 1]");  // :578-580
  TORCH_CHECK(lifecycle_logits.dim() == 3 && lifecycle_logits.size(0) == batch &&
                  lifecycle_logits.size(1) == slots,
              "lifecycle_logits must have shape [batch, slots, lifecycles]");  // :581-585
  TORCH_CHECK(selected.sizes() == at::IntArrayRef({batch, slots}),
              "selected must have shape [batch, slots]");  // :586-588
  TORCH_CHECK(selected.scalar_type() == at::kBool, "selected must use torch.bool");  // :589-591
  TORCH_CHECK(semantic_indices.dim() == 1 && semantic_indices.scalar_type() == at::kLong,
              "semantic_indices must be a one-dimensional int64 tensor");  // :592-595
  TORCH_CHECK(lifecycle_logits.size(-1) > 0, "lifecycle_logits must be non-empty");
  for (const at::Tensor* t : {&thought_semantic, &role_logits, &uncertainty, &noise_delta,
                              &lifecycle_logits})
    TORCH_CHECK(t->is_floating_point(), "snapshot inputs must use floating dtypes");
  if (semantic_indices.device().is_cpu() && semantic_indices.numel() != 0) {
    // host-resident indices are validated here without any device sync (:596-601)
    auto idx = semantic_indices.contiguous();
    const auto* p = idx.data_ptr<std::int64_t>();
    for (std::int64_t k = 0; k < idx.numel(); ++k)
      TORCH_CHECK(p[k] >= 0 && p[k] < hidden,
                  "semantic_indices contain values outside semantic width");
  }
  same_device("materialize_cell_snapshot", {&thought_semantic, &role_logits, &uncertainty,
                                            &noise_delta, &lifecycle_logits, &selected});
  const auto width = 4 + role_logits.size(-1) + semantic_indices.numel();
  auto out = at::empty({batch, slots, width}, thought_semantic.options().dtype(at::kFloat));
  if (backend == Backend::kMeta) return out;
  if (backend == Backend::kCpu) detail::no_cpu_backend("materialize_cell_snapshot");
  if (batch * slots == 0) return out;
  const c10::cuda::CUDAGuard guard(thought_semantic.device());
  auto sem = thought_semantic.contiguous();
  auto roles = role_logits.contiguous();
  auto unc = uncertainty.contiguous();
  auto noise = noise_delta.contiguous();
  auto life = lifecycle_logits.contiguous();
  auto sel = selected.contiguous();
  auto idx = semantic_indices.to(sem.device()).contiguous();  // :610
  check_result(cid_materialize_cell_snapshot(
                   dt(sem), sem.data_ptr(), hidden, dt(roles), roles.data_ptr(), roles.size(-1),
                   dt(unc), unc.data_ptr(), dt(noise), noise.data_ptr(), dt(life),
                   life.data_ptr(), life.size(-1),
                   reinterpret_cast<const std::uint8_t*>(sel.data_ptr<bool>()),
                   idx.numel() ? idx.data_ptr<std::int64_t>() : nullptr, idx.numel(),
                   batch * slots, out.data_ptr<float>(), detail::status_word(sem.device()),
                   stream_of(sem)),
               "materialize_cell_snapshot");
  return out;
}

}  // namespace cid::engine
