// Host entry points of the B200 build of cid-engine.
//
// The functions keep the names and signatures of the reference's public
// header (csrc/include/cid_engine/ops.hpp:9-107 of fwerkor/cid-engine
// v1.1.0).  Each operator validates its arguments exactly once (with the
// reference's error messages) and then, depending on the dispatch key,
//   * CUDA: enqueues the sm_100a kernels through the C ABI
//     (include/cid_engine_b200.h) on the current stream of the inputs' device;
//   * Meta: returns empty outputs of the right shapes and dtypes;
//   * CPU:  raises — this library has no CPU backend.
#pragma once

#include <ATen/ATen.h>

#include <cstdint>
#include <optional>
#include <tuple>

namespace cid::engine {

enum class Backend { kCuda, kMeta, kCpu };

using Tensor3 = std::tuple<at::Tensor, at::Tensor, at::Tensor>;
using Tensor4 = std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor>;
using Tensor6 =
    std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor>;
using Tensor7 = std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                           at::Tensor, at::Tensor>;

at::Tensor live_slot_occupancy(Backend backend, const at::Tensor& slot_occupancy,
                               const std::optional<at::Tensor>& lifecycle_features,
                               std::int64_t retired_index);

at::Tensor prefix_allocation_mask(Backend backend, const at::Tensor& occupancy,
                                  const at::Tensor& allocation_logits, double threshold,
                                  std::int64_t max_allocations);

at::Tensor batched_linear_assignment(Backend backend, const at::Tensor& costs,
                                     const at::Tensor& row_counts);

Tensor6 rollout_slot_transition(Backend backend, const at::Tensor& occupancy,
                                const at::Tensor& allocation_logits,
                                const at::Tensor& lifecycle_logits,
                                const at::Tensor& revision_logits,
                                const at::Tensor& input_lifecycle, double threshold,
                                std::int64_t max_allocations, std::int64_t retired_index);

Tensor7 rollout_slot_transition_with_live(Backend backend, const at::Tensor& occupancy,
                                          const at::Tensor& allocation_logits,
                                          const at::Tensor& lifecycle_logits,
                                          const at::Tensor& revision_logits,
                                          const at::Tensor& input_lifecycle, double threshold,
                                          std::int64_t max_allocations,
                                          std::int64_t retired_index);

Tensor3 thought_corrupt_from_epsilon(Backend backend, const at::Tensor& semantic,
                                     const at::Tensor& timesteps, const at::Tensor& occupancy,
                                     const at::Tensor& epsilon);

Tensor4 display_corrupt_from_random(Backend backend, const at::Tensor& token_ids,
                                    const at::Tensor& timesteps, const at::Tensor& eligible_mask,
                                    const at::Tensor& corruption_random,
                                    const std::optional<at::Tensor>& replacement_random,
                                    const std::optional<at::Tensor>& replacement_offsets,
                                    std::int64_t mask_token_id,
                                    const std::optional<std::int64_t>& eos_token_id,
                                    std::int64_t vocab_size, double replacement_fraction);

Tensor4 masked_diffusion_corrupt_from_random(Backend backend, const at::Tensor& clean_ids,
                                             const at::Tensor& ratio_random,
                                             const at::Tensor& mask_random,
                                             std::int64_t mask_token_id, double min_mask_ratio,
                                             double max_mask_ratio);

Tensor3 display_token_statistics(Backend backend, const at::Tensor& token_ids,
                                 const at::Tensor& logits);

Tensor3 display_token_statistics_with_repetition(
    Backend backend, const at::Tensor& token_ids, const at::Tensor& logits,
    std::int64_t mask_token_id, const std::optional<std::int64_t>& eos_token_id,
    double repetition_score_multiplier);

at::Tensor refine_display_from_statistics(
    Backend backend, const at::Tensor& token_ids, const at::Tensor& confidence,
    const at::Tensor& predicted, const at::Tensor& current_confidence,
    std::int64_t mask_token_id, const std::optional<std::int64_t>& eos_token_id,
    double reveal_fraction, double revision_fraction, double revision_margin);

at::Tensor materialize_cell_snapshot(Backend backend, const at::Tensor& thought_semantic,
                                     const at::Tensor& role_logits,
                                     const at::Tensor& uncertainty,
                                     const at::Tensor& noise_delta,
                                     const at::Tensor& lifecycle_logits,
                                     const at::Tensor& selected,
                                     const at::Tensor& semantic_indices);

// Vocabulary-parallel statistics (additive operators of this library).
at::Tensor display_shard_records(Backend backend, const at::Tensor& token_ids,
                                 const at::Tensor& logits_shard, std::int64_t vocab_offset,
                                 std::int64_t total_vocab);
Tensor3 display_combine_records(Backend backend, const at::Tensor& records,
                                const at::Tensor& token_ids, at::IntArrayRef shard_offsets);

// LM head fused with the display statistics (additive operator of this
// build): display_token_statistics(token_ids, hidden @ weight^T) without
// writing the logits.
Tensor3 lm_head_display_statistics(Backend backend, const at::Tensor& token_ids,
                                   const at::Tensor& hidden, const at::Tensor& weight,
                                   bool round_bf16);
// The per-rank half of a vocabulary-parallel LM head: shard records [rows, 4]
// (int32) of hidden @ weight_shard^T for global columns starting at vocab_offset.
at::Tensor lm_head_shard_records(Backend backend, const at::Tensor& token_ids,
                                 const at::Tensor& hidden, const at::Tensor& weight_shard,
                                 std::int64_t vocab_offset, std::int64_t total_vocab,
                                 bool round_bf16);

// Device status word (CID_STATUS_* bits) of `device`; read() synchronises.
std::int64_t read_device_status(std::int64_t device, bool reset);

// Shared helpers of the host translation units.
namespace detail {
int dtype_code(at::ScalarType t);
void check_result(int rc, const char* op);
std::uint32_t* status_word(const at::Device& device);
[[noreturn]] void no_cpu_backend(const char* op);
}  // namespace detail

}  // namespace cid::engine
