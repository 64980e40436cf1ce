// Operator registration.  The schema strings are the reference's stable
// operator ABI (csrc/registration.cpp:5-49 of fwerkor/cid-engine v1.1.0) and
// are kept byte-for-byte identical so that callers of
// torch.ops.cid_engine.<op> need no change.  Two operators are added for the
// vocabulary-parallel statistics.
//
// Kernels are registered per dispatch key (the reference registers
// CompositeImplicitAutograd ATen implementations plus CUDA overrides):
//   CUDA -> sm_100a kernels, Meta -> shape functions, CPU -> validation and
//   a clear error (this library has no CPU backend).
#include <torch/library.h>

#include "cid_engine/ops.hpp"

namespace cid::engine {
namespace {

template <Backend B>
at::Tensor live_impl(const at::Tensor& occ, const std::optional<at::Tensor>& life, std::int64_t r) {
  return live_slot_occupancy(B, occ, life, r);
}
template <Backend B>
at::Tensor prefix_impl(const at::Tensor& occ, const at::Tensor& lg, double thr, std::int64_t n) {
  return prefix_allocation_mask(B, occ, lg, thr, n);
}
template <Backend B>
at::Tensor assignment_impl(const at::Tensor& costs, const at::Tensor& counts) {
  return batched_linear_assignment(B, costs, counts);
}
template <Backend B>
Tensor6 rollout_impl(const at::Tensor& occ, const at::Tensor& al, const at::Tensor& lc,
                     const at::Tensor& rv, const at::Tensor& il, double thr, std::int64_t n,
                     std::int64_t r) {
  return rollout_slot_transition(B, occ, al, lc, rv, il, thr, n, r);
}
template <Backend B>
Tensor7 rollout_live_impl(const at::Tensor& occ, const at::Tensor& al, const at::Tensor& lc,
                          const at::Tensor& rv, const at::Tensor& il, double thr, std::int64_t n,
                          std::int64_t r) {
  return rollout_slot_transition_with_live(B, occ, al, lc, rv, il, thr, n, r);
}
template <Backend B>
Tensor3 thought_impl(const at::Tensor& s, const at::Tensor& t, const at::Tensor& o,
                     const at::Tensor& e) {
  return thought_corrupt_from_epsilon(B, s, t, o, e);
}
template <Backend B>
Tensor4 display_corrupt_impl(const at::Tensor& ids, const at::Tensor& ts, const at::Tensor& el,
                             const at::Tensor& cr, const std::optional<at::Tensor>& rr,
                             const std::optional<at::Tensor>& ro, std::int64_t mask,
                             std::optional<std::int64_t> eos, std::int64_t vocab, double frac) {
  return display_corrupt_from_random(B, ids, ts, el, cr, rr, ro, mask, eos, vocab, frac);
}
template <Backend B>
Tensor4 masked_impl(const at::Tensor& c, const at::Tensor& rr, const at::Tensor& mr,
                    std::int64_t mask, double lo, double hi) {
  return masked_diffusion_corrupt_from_random(B, c, rr, mr, mask, lo, hi);
}
template <Backend B>
Tensor3 stats_impl(const at::Tensor& ids, const at::Tensor& lg) {
  return display_token_statistics(B, ids, lg);
}
template <Backend B>
Tensor3 stats_rep_impl(const at::Tensor& ids, const at::Tensor& lg, std::int64_t mask,
                       std::optional<std::int64_t> eos, double mult) {
  return display_token_statistics_with_repetition(B, ids, lg, mask, eos, mult);
}
template <Backend B>
at::Tensor refine_impl(const at::Tensor& ids, const at::Tensor& conf, const at::Tensor& pred,
                       const at::Tensor& cur, std::int64_t mask, std::optional<std::int64_t> eos,
                       double reveal, double revision, double margin) {
  return refine_display_from_statistics(B, ids, conf, pred, cur, mask, eos, reveal, revision,
                                        margin);
}
template <Backend B>
at::Tensor snapshot_impl(const at::Tensor& s, const at::Tensor& r, const at::Tensor& u,
                         const at::Tensor& n, const at::Tensor& l, const at::Tensor& sel,
                         const at::Tensor& idx) {
  return materialize_cell_snapshot(B, s, r, u, n, l, sel, idx);
}
template <Backend B>
at::Tensor shard_records_impl(const at::Tensor& ids, const at::Tensor& lg, std::int64_t off,
                              std::int64_t total) {
  return display_shard_records(B, ids, lg, off, total);
}
template <Backend B>
Tensor3 combine_records_impl(const at::Tensor& rec, const at::Tensor& ids, at::IntArrayRef offs) {
  return display_combine_records(B, rec, ids, offs);
}

template <Backend B>
Tensor3 lm_head_impl(const at::Tensor& ids, const at::Tensor& hidden, const at::Tensor& weight,
                     bool round_bf16) {
  return lm_head_display_statistics(B, ids, hidden, weight, round_bf16);
}

template <Backend B>
at::Tensor lm_head_shard_impl(const at::Tensor& ids, const at::Tensor& hidden,
                              const at::Tensor& weight, std::int64_t off, std::int64_t total,
                              bool round_bf16) {
  return lm_head_shard_records(B, ids, hidden, weight, off, total, round_bf16);
}

template <Backend B>
void register_all(torch::Library& m) {
  m.impl("live_slot_occupancy", TORCH_FN(live_impl<B>));
  m.impl("prefix_allocation_mask", TORCH_FN(prefix_impl<B>));
  m.impl("batched_linear_assignment", TORCH_FN(assignment_impl<B>));
  m.impl("rollout_slot_transition", TORCH_FN(rollout_impl<B>));
  m.impl("rollout_slot_transition_with_live", TORCH_FN(rollout_live_impl<B>));
  m.impl("thought_corrupt_from_epsilon", TORCH_FN(thought_impl<B>));
  m.impl("display_corrupt_from_random", TORCH_FN(display_corrupt_impl<B>));
  m.impl("masked_diffusion_corrupt_from_random", TORCH_FN(masked_impl<B>));
  m.impl("display_token_statistics", TORCH_FN(stats_impl<B>));
  m.impl("display_token_statistics_with_repetition", TORCH_FN(stats_rep_impl<B>));
  m.impl("refine_display_from_statistics", TORCH_FN(refine_impl<B>));
  m.impl("materialize_cell_snapshot", TORCH_FN(snapshot_impl<B>));
  m.impl("display_shard_records", TORCH_FN(shard_records_impl<B>));
  m.impl("display_combine_records", TORCH_FN(combine_records_impl<B>));
  m.impl("lm_head_display_statistics", TORCH_FN(lm_head_impl<B>));
  m.impl("lm_head_shard_records", TORCH_FN(lm_head_shard_impl<B>));
}

}  // namespace
}  // namespace cid::engine

TORCH_LIBRARY(cid_engine, m) {
  m.def(
      "live_slot_occupancy(Tensor slot_occupancy, Tensor? lifecycle_features, "
      "int retired_index) -> Tensor");
  m.def(
      "prefix_allocation_mask(Tensor occupancy, Tensor allocation_logits, "
      "float threshold, int max_allocations) -> Tensor");
  m.def("batched_linear_assignment(Tensor costs, Tensor row_counts) -> Tensor");
  m.def(
      "rollout_slot_transition(Tensor occupancy, Tensor allocation_logits, "
      "Tensor lifecycle_logits, Tensor revision_logits, Tensor input_lifecycle, "
      "float threshold, int max_allocations, int retired_index) "
      "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def(
      "thought_corrupt_from_epsilon(Tensor semantic, Tensor timesteps, "
      "Tensor occupancy, Tensor epsilon) -> (Tensor, Tensor, Tensor)");
  m.def(
      "display_corrupt_from_random(Tensor token_ids, Tensor timesteps, "
      "Tensor eligible_mask, Tensor corruption_random, Tensor? replacement_random, "
      "Tensor? replacement_offsets, int mask_token_id, int? eos_token_id, "
      "int vocab_size, float replacement_fraction) "
      "-> (Tensor, Tensor, Tensor, Tensor)");
  m.def(
      "masked_diffusion_corrupt_from_random(Tensor clean_ids, "
      "Tensor ratio_random, Tensor mask_random, int mask_token_id, "
      "float min_mask_ratio, float max_mask_ratio) "
      "-> (Tensor, Tensor, Tensor, Tensor)");
  m.def(
      "display_token_statistics(Tensor token_ids, Tensor logits) "
      "-> (Tensor, Tensor, Tensor)");
  m.def(
      "display_token_statistics_with_repetition(Tensor token_ids, Tensor logits, "
      "int mask_token_id, int? eos_token_id, float repetition_score_multiplier) "
      "-> (Tensor, Tensor, Tensor)");
  m.def(
      "refine_display_from_statistics(Tensor token_ids, Tensor confidence, "
      "Tensor predicted, Tensor current_confidence, int mask_token_id, "
      "int? eos_token_id, float reveal_fraction, float revision_fraction, "
      "float revision_margin) -> Tensor");
  m.def(
      "materialize_cell_snapshot(Tensor thought_semantic, Tensor role_logits, "
      "Tensor uncertainty, Tensor noise_delta, Tensor lifecycle_logits, "
      "Tensor selected, Tensor semantic_indices) -> Tensor");
  // additive: the decode step's slot rollout with the live occupancy of the
  // next state, one kernel
  m.def(
      "rollout_slot_transition_with_live(Tensor occupancy, Tensor allocation_logits, "
      "Tensor lifecycle_logits, Tensor revision_logits, Tensor input_lifecycle, "
      "float threshold, int max_allocations, int retired_index) "
      "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  // additive: vocabulary-parallel statistics
  m.def(
      "display_shard_records(Tensor token_ids, Tensor logits_shard, int vocab_offset, "
      "int total_vocab) -> Tensor");
  m.def(
      "display_combine_records(Tensor records, Tensor token_ids, int[] shard_offsets) "
      "-> (Tensor, Tensor, Tensor)");
  // additive: LM head fused with the display statistics
  m.def(
      "lm_head_display_statistics(Tensor token_ids, Tensor hidden, Tensor weight, "
      "bool round_bf16=True) -> (Tensor, Tensor, Tensor)");
  m.def(
      "lm_head_shard_records(Tensor token_ids, Tensor hidden, Tensor weight_shard, "
      "int vocab_offset, int total_vocab, bool round_bf16=True) -> Tensor");
}

TORCH_LIBRARY_IMPL(cid_engine, CUDA, m) {
  cid::engine::register_all<cid::engine::Backend::kCuda>(m);
}
TORCH_LIBRARY_IMPL(cid_engine, Meta, m) {
  cid::engine::register_all<cid::engine::Backend::kMeta>(m);
}
TORCH_LIBRARY_IMPL(cid_engine, CPU, m) {
  cid::engine::register_all<cid::engine::Backend::kCpu>(m);
}
