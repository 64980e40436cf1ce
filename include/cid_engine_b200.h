/*
 * cid_engine_b200.h — C ABI of the B200 (sm_100a) display-refinement kernels.
 *
 * Plain pointers, sizes and enums; no torch or C++ types.  Every entry point
 * is asynchronous: it validates its arguments on the host, enqueues its
 * kernel(s) on `stream` (a cudaStream_t passed as void*, NULL = legacy default
 * stream) for the device that is current on the calling thread, and returns
 * a cid_result_t.  Device pointers must belong to that device.
 *
 * Each entry point replaces one reference operator (fwerkor/cid-engine
 * v1.1.0); the reference interface is cited beside it.  Argument meaning and
 * output semantics are those of the reference CPU backend.
 *
 * Host-side validation.  Before its first CUDA call every entry point checks,
 * in this order: its dtype codes (CID_ERR_UNSUPPORTED_DTYPE); its scalar
 * arguments and extents (CID_ERR_INVALID_ARGUMENT) — negative extents, row
 * or batch counts above 2^31 - 1, arrays of more than 2^58 elements, element
 * counts that overflow int64; the alignment of every non-NULL pointer to its
 * element size, or to 16 bytes where an entry point says so
 * (CID_ERR_MISALIGNED); then it returns CID_OK when there is no work, and
 * otherwise rejects a NULL pointer for any array of non-zero extent that it
 * reads or writes (CID_ERR_INVALID_ARGUMENT; `status` may always be NULL).
 * Host arrays (shard offsets, inbox lists, IPC handles) are read only within
 * their documented extents, after the extent itself has been checked.
 *
 * Device-side status.  Conditions that the reference CPU backend turns into
 * exceptions but that a device kernel cannot raise without a host sync (an
 * out-of-range token id, a snapshot index outside the semantic width) are
 * reported by OR-ing CID_STATUS_* bits into an optional device word
 * `status` (may be NULL); the affected outputs are written as NaN (floats)
 * and no out-of-bounds access is made.
 */
#ifndef CID_ENGINE_B200_H
#define CID_ENGINE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CID_API __attribute__((visibility("default")))
#else
#define CID_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CID_ENGINE_B200_ABI_VERSION 1

typedef enum cid_dtype {
  CID_DTYPE_F32 = 0,
  CID_DTYPE_F64 = 1,
  CID_DTYPE_F16 = 2,
  CID_DTYPE_BF16 = 3,
  CID_DTYPE_BOOL = 4,
  CID_DTYPE_I64 = 5,
  CID_DTYPE_I32 = 6,
  CID_DTYPE_U8 = 7,
  CID_DTYPE_I8 = 8,
  CID_DTYPE_I16 = 9,
  /* Not dtypes: these two make every 32-bit int a value of the type, so an
   * unknown code from a caller is a defined value that the entry points
   * reject with CID_ERR_UNSUPPORTED_DTYPE. */
  CID_DTYPE_RANGE_MIN_ = -0x7fffffff - 1,
  CID_DTYPE_RANGE_MAX_ = 0x7fffffff
} cid_dtype_t;

typedef enum cid_result {
  CID_OK = 0,
  CID_ERR_INVALID_ARGUMENT = 1,
  CID_ERR_UNSUPPORTED_DTYPE = 2,
  CID_ERR_LAUNCH = 3,
  CID_ERR_MISALIGNED = 4,
  CID_ERR_CUDA = 5,
  CID_ERR_SCRATCH_LIMIT = 6
} cid_result_t;

/* Bits OR-ed into the optional device status word. */
#define CID_STATUS_TOKEN_ID_OUT_OF_RANGE 0x1u
#define CID_STATUS_SEMANTIC_INDEX_OUT_OF_RANGE 0x2u
#define CID_STATUS_REPETITION_ID_OUT_OF_RANGE 0x4u
#define CID_STATUS_ASSIGNMENT_INVALID 0x8u
/* A bounded wait of the LM-head kernel ran out (its outputs are invalid). */
#define CID_STATUS_LM_HEAD_TIMEOUT 0x10u
/* A rank's records of this epoch did not arrive in a peer exchange's wait
 * (its statistics are NaN). */
#define CID_STATUS_PEER_TIMEOUT 0x20u
/* A rank ran two or more epochs ahead of this rank's combine in a peer
 * exchange (it gave up waiting on this rank earlier), so this rank's inbox
 * may hold a later step's records: the step's statistics are invalid. */
#define CID_STATUS_PEER_OUT_OF_STEP 0x40u

CID_API int cid_abi_version(void);
CID_API const char* cid_result_string(int result);
/* Message of the last CUDA error seen by this thread inside the library. */
CID_API const char* cid_last_cuda_error(void);

/* ---------------------------------------------------------------------- */
/* Display statistics                                                      */
/* ---------------------------------------------------------------------- */

/* display_token_statistics — replaces
 *   csrc/registration.cpp:33-35 (schema), csrc/cpu/display_stats.cpp:54-126
 *   (CPU semantics), csrc/cuda/display_stats.cu:168-220 (CUDA launcher).
 * logits: rows x vocab of `dtype` (F32/F64/F16/BF16), row r at
 *   logits + r*row_stride elements, unit stride along the vocabulary.
 * Outputs per row: confidence = max softmax probability, predicted = argmax
 *   (first NaN, else lowest index of the maximum), current_confidence =
 *   softmax probability of token_ids[r].  rows may be 0. */
CID_API int cid_display_token_statistics(cid_dtype_t dtype, const void* logits,
                                 int64_t row_stride, const int64_t* token_ids,
                                 int64_t rows, int64_t vocab, float* confidence,
                                 int64_t* predicted, float* current_confidence,
                                 uint32_t* status, void* stream);

/* display_token_statistics_with_repetition — replaces
 *   csrc/registration.cpp:36-39, csrc/ops.cpp:477-552,
 *   csrc/cuda/display_stats.cu:222-283.
 * token_ids/logits as above with rows = batch*tokens (row b*tokens+p).
 * has_eos = 0 means eos_token_id is None.  multiplier in (0, 1]. */
CID_API int cid_display_token_statistics_with_repetition(
    cid_dtype_t dtype, const void* logits, int64_t row_stride,
    const int64_t* token_ids, int64_t batch, int64_t tokens, int64_t vocab,
    int64_t mask_token_id, int has_eos, int64_t eos_token_id,
    double multiplier, float* confidence, int64_t* predicted,
    float* current_confidence, uint32_t* status, void* stream);

/* Vocabulary-parallel statistics.  A rank holding columns
 * [vocab_offset, vocab_offset + shard_vocab) of a total_vocab-wide row
 * writes one 16-byte record per row; the records of all ranks (gathered in
 * rank order, ranks holding ascending contiguous ranges) are merged by
 * cid_display_combine_records into the unsharded statistics.  This is the
 * multi-GPU form of display_token_statistics (no reference counterpart
 * beyond the operator it decomposes). */
typedef struct cid_shard_record {
  float max_logit;   /* shard maximum (ignores NaN) */
  float sum_exp;     /* sum over the shard of exp(x - max_logit) */
  int32_t index;     /* global column of the first maximum; bit 31 set
                        when the shard holds a NaN, the low bits then give
                        the global column of its first NaN */
  float current;     /* logit of token_ids[r] when this shard owns it */
} cid_shard_record_t;

CID_API int cid_display_shard_records(cid_dtype_t dtype, const void* logits,
                              int64_t row_stride, const int64_t* token_ids,
                              int64_t rows, int64_t shard_vocab,
                              int64_t vocab_offset, int64_t total_vocab,
                              cid_shard_record_t* records, uint32_t* status,
                              void* stream);

/* records: world x rows (rank-major), world <= 256.  shard_offsets: world+1
 * ascending column offsets within [0, 2^31 - 1] on the HOST (shard r owns
 * [offsets[r], offsets[r+1])). */
/* Merges records [world][rows] of ascending column ranges shard_offsets_host
 * (world + 1 host values) into one record per row of their union, as
 * cid_display_shard_records would produce for the concatenated range (no
 * reference counterpart: the merge inside one GPU of the vocabulary-parallel
 * statistics, used by cid_lm_head_shard_records). */
CID_API int cid_display_merge_records(const cid_shard_record_t* records, int world,
                        const int64_t* shard_offsets_host, const int64_t* token_ids,
                        int64_t rows, cid_shard_record_t* merged, void* stream);

CID_API int cid_display_combine_records(const cid_shard_record_t* records, int world,
                                const int64_t* shard_offsets_host,
                                const int64_t* token_ids, int64_t rows,
                                float* confidence, int64_t* predicted,
                                float* current_confidence, uint32_t* status,
                                void* stream);

/* ---------------------------------------------------------------------- */
/* Refinement policy                                                       */
/* ---------------------------------------------------------------------- */

/* refine_display_from_statistics — replaces csrc/registration.cpp:40-44 and
 * csrc/refine.cpp:222-429 (which copies to the host and back every call);
 * here one CTA per row runs the whole policy on the device.
 * All arrays batch x tokens, contiguous. `out` must not alias the inputs. */
CID_API int cid_refine_display(const int64_t* token_ids, const float* confidence,
                       const int64_t* predicted,
                       const float* current_confidence, int64_t batch,
                       int64_t tokens, int64_t mask_token_id, int has_eos,
                       int64_t eos_token_id, double reveal_fraction,
                       double revision_fraction, double revision_margin,
                       int64_t* out, void* stream);

/* ---------------------------------------------------------------------- */
/* Thought-slot state                                                      */
/* ---------------------------------------------------------------------- */

/* prefix_allocation_mask — replaces csrc/registration.cpp:9-11,
 * csrc/ops.cpp:41-65, csrc/cuda/prefix_allocation.cu:81-132.
 * occupancy: batch x slots of occ_dtype (any), element (b,s) at
 *   occupancy + b*occ_row_stride + s*occ_col_stride;
 * logits: same shape of logit_dtype (F32/F64/F16/BF16), strided likewise;
 * out: batch x slots bool (uint8), contiguous. */
CID_API int cid_prefix_allocation_mask(cid_dtype_t occ_dtype, const void* occupancy,
                               int64_t occ_row_stride, int64_t occ_col_stride,
                               cid_dtype_t logit_dtype, const void* logits,
                               int64_t logit_row_stride,
                               int64_t logit_col_stride, int64_t batch,
                               int64_t slots, double threshold,
                               int64_t max_allocations, uint8_t* out,
                               void* stream);

/* rollout_slot_transition — replaces csrc/registration.cpp:14-18,
 * csrc/ops.cpp:184-256, csrc/cuda/rollout_state.cu:134-281.
 * allocation_logits (batch x slots), lifecycle_logits and input_lifecycle
 * (batch x slots x lifecycles), revision_logits (batch x slots x revisions):
 * contiguous, all of `dtype`.  Outputs contiguous batch x slots. */
CID_API int cid_rollout_slot_transition(
    cid_dtype_t occ_dtype, const void* occupancy, cid_dtype_t dtype,
    const void* allocation_logits, const void* lifecycle_logits,
    const void* revision_logits, const void* input_lifecycle, int64_t batch,
    int64_t slots, int64_t lifecycles, int64_t revisions, double threshold,
    int64_t max_allocations, int64_t retired_index, uint8_t* next_occupancy,
    int64_t* lifecycle_indices, int64_t* revision_indices,
    int64_t* input_lifecycle_indices, uint8_t* input_lifecycle_present,
    uint8_t* live_slots, void* stream);

/* cid_rollout_slot_transition plus, in the same launch, the live occupancy
 * of the next state: live_slot_occupancy (csrc/ops.cpp:12-39) of
 * next_occupancy (as a 0/1 value of live_dtype, the lifecycle logits'
 * dtype) with lifecycle_logits and retired_index, into live_occupancy
 * (batch x slots of live_dtype).  The decode step's slot rollout followed by
 * its live occupancy (csrc/ops.cpp:184-256 then :12-39) in one kernel. */
CID_API int cid_rollout_slot_transition_live(
    cid_dtype_t occ_dtype, const void* occupancy, cid_dtype_t dtype,
    const void* allocation_logits, const void* lifecycle_logits, const void* revision_logits,
    const void* input_lifecycle, int64_t batch, int64_t slots, int64_t lifecycles,
    int64_t revisions, double threshold, int64_t max_allocations, int64_t retired_index,
    uint8_t* next_occupancy, int64_t* lifecycle_indices, int64_t* revision_indices,
    int64_t* input_lifecycle_indices, uint8_t* input_lifecycle_present, uint8_t* live_slots,
    cid_dtype_t live_dtype, void* live_occupancy, void* stream);

/* live_slot_occupancy — replaces csrc/registration.cpp:6-8 and
 * csrc/ops.cpp:12-39.  occupancy: rows (= batch*slots) of `dtype`;
 * lifecycle: rows x features of `dtype` or NULL; out: rows of `dtype`. */
CID_API int cid_live_slot_occupancy(cid_dtype_t dtype, const void* occupancy,
                            const void* lifecycle, int64_t rows,
                            int64_t features, int64_t retired_index, void* out,
                            void* stream);

/* materialize_cell_snapshot — replaces csrc/registration.cpp:45-48,
 * csrc/ops.cpp:556-615, csrc/cuda/materialize_snapshot.cu:71-184.
 * rows = batch*slots; every input contiguous with its own dtype; selected
 * bool; indices int64 on the device; out rows x (4+roles+nindices) f32. */
CID_API int cid_materialize_cell_snapshot(
    cid_dtype_t sem_dtype, const void* semantic, int64_t hidden,
    cid_dtype_t role_dtype, const void* roles, int64_t nroles,
    cid_dtype_t unc_dtype, const void* uncertainty, cid_dtype_t noise_dtype,
    const void* noise_delta, cid_dtype_t life_dtype, const void* lifecycle,
    int64_t lifecycles, const uint8_t* selected, const int64_t* indices,
    int64_t nindices, int64_t rows, float* out, uint32_t* status,
    void* stream);

/* batched_linear_assignment — replaces csrc/registration.cpp:12-13,
 * csrc/ops.cpp:68-175, csrc/cuda/linear_assignment.cu.
 * costs: batch x rows x columns of cost_dtype (read as float32, solved in
 * double), rows <= columns <= 16; row_counts: batch int64 (active rows);
 * out: batch x rows int64, the column assigned to each active row, -1
 * elsewhere.  A row count outside [0, rows], or costs for which the search
 * cannot complete (non-finite), leave that batch element at -1 and set
 * CID_STATUS_ASSIGNMENT_INVALID. */
CID_API int cid_batched_linear_assignment(cid_dtype_t cost_dtype,
                                          const void* costs,
                                          const int64_t* row_counts,
                                          int64_t batch, int64_t rows,
                                          int64_t columns, int64_t* out,
                                          uint32_t* status, void* stream);

/* ---------------------------------------------------------------------- */
/* Training corruption                                                     */
/* ---------------------------------------------------------------------- */

/* Scratch bytes cid_masked_diffusion_corrupt needs in `workspace`. */
CID_API size_t cid_masked_diffusion_workspace_bytes(int64_t batch);

/* masked_diffusion_corrupt_from_random — replaces
 * csrc/registration.cpp:28-32, csrc/ops.cpp:394-444,
 * csrc/cuda/masked_diffusion.cu:100-170.
 * clean_ids batch x tokens int64; ratio_random batch (F32); mask_random
 * batch x tokens (F32); outputs corrupted (int64), masked (bool), ratio
 * (batch f32), metrics (2 f32: mean mask, mean ratio; summed in a fixed
 * order, so repeated calls give identical metrics).  workspace: device
 * scratch of cid_masked_diffusion_workspace_bytes(batch) bytes, 16-byte
 * aligned, contents need not be initialised.
 * A call on a stream that is being captured into a CUDA graph is captured
 * as one kernel (eagerly: two) once an eager call on the same device has
 * run: it takes one of 4096 accumulator slots per device held in the
 * library's device image, which the captured kernel keeps for the life of
 * the process and clears after every run.  Outputs are bit-identical either
 * way.  Two executable instances of one such graph must not run at the
 * same time; replays of one instance are ordered by CUDA.  When the slots
 * are spent, or batch >= 2^24, calls are captured as two kernels over the
 * workspace. */
CID_API int cid_masked_diffusion_corrupt(const int64_t* clean_ids,
                                 const float* ratio_random,
                                 const float* mask_random, int64_t batch,
                                 int64_t tokens, int64_t mask_token_id,
                                 double min_mask_ratio, double max_mask_ratio,
                                 int64_t* corrupted, uint8_t* masked,
                                 float* ratio, float* metrics, void* workspace,
                                 void* stream);

/* Allocation-free masked diffusion.  No counterpart in the reference: it is
 * an extra way to call cid_masked_diffusion_corrupt for callers that cannot
 * allocate device memory for a workspace — a host program that reserves all
 * device memory for its own pool and forbids third-party cudaMalloc, a
 * serving loop that must not pay cudaMalloc's latency and implicit
 * synchronisation per request, or an FFI binding with no device allocator.
 * Same arguments and outputs as cid_masked_diffusion_corrupt minus the
 * workspace; the caller still passes every input and output.  Scratch is a
 * fixed array inside the library's device image, CID_NO_ALLOC_MAX_BATCH rows
 * (512 KiB), held by every GPU that loads the library until the process
 * exits; batch > CID_NO_ALLOC_MAX_BATCH returns CID_ERR_SCRATCH_LIMIT.  The
 * first call on a device looks up the array's device address (a
 * cudaGetSymbolAddress with that device current), so make that first call
 * before any stream capture.  The address is cached per device for the
 * device's primary context (the one the CUDA runtime uses by default): a
 * caller that runs the library in a context of its own (cuCtxCreate), or
 * calls it after cudaDeviceReset in the same process, would be handed a
 * stale address and must use cid_masked_diffusion_corrupt instead.  Calls
 * on one device share the array: calls that overlap on the GPU (on
 * different streams) race on it.  Nothing in it needs clearing between
 * calls. */
#define CID_NO_ALLOC_MAX_BATCH 65536
CID_API int cid_masked_diffusion_corrupt_no_alloc(
    const int64_t* clean_ids, const float* ratio_random,
    const float* mask_random, int64_t batch, int64_t tokens,
    int64_t mask_token_id, double min_mask_ratio, double max_mask_ratio,
    int64_t* corrupted, uint8_t* masked, float* ratio, float* metrics,
    void* stream);

/* thought_corrupt_from_epsilon — replaces csrc/registration.cpp:19-21,
 * csrc/ops.cpp:258-290, csrc/cuda/thought_corruption.cu:72-157.
 * semantic/epsilon/corrupted/masked_epsilon: rows x hidden of sem_dtype;
 * timesteps: rows of t_dtype; occupancy: rows of occ_dtype; local_noise:
 * rows of sem_dtype.  All contiguous. */
CID_API int cid_thought_corrupt(cid_dtype_t sem_dtype, const void* semantic,
                        cid_dtype_t t_dtype, const void* timesteps,
                        cid_dtype_t occ_dtype, const void* occupancy,
                        const void* epsilon, int64_t rows, int64_t hidden,
                        void* corrupted, void* local_noise,
                        void* masked_epsilon, void* stream);

/* display_corrupt_from_random — replaces csrc/registration.cpp:22-27,
 * csrc/ops.cpp:292-391, csrc/cuda/display_corruption.cu.
 * token_ids batch x tokens int64; timesteps batch (t_dtype); eligible
 * batch x tokens (elig_dtype); corruption_random and replacement_random
 * batch x tokens (float dtypes; replacement_* may be NULL when
 * replacement_fraction == 0); replacement_offsets int64.  Outputs int64
 * corrupted and labels, bool masked and replaced. */
CID_API int cid_display_corrupt(const int64_t* token_ids, cid_dtype_t t_dtype,
                        const void* timesteps, cid_dtype_t elig_dtype,
                        const void* eligible, cid_dtype_t rand_dtype,
                        const void* corruption_random, cid_dtype_t repl_dtype,
                        const void* replacement_random,
                        const int64_t* replacement_offsets, int64_t batch,
                        int64_t tokens, int64_t mask_token_id, int has_eos,
                        int64_t eos_token_id, int64_t vocab_size,
                        double replacement_fraction, int64_t* corrupted,
                        int64_t* labels, uint8_t* masked, uint8_t* replaced,
                        void* stream);

/* ---------------------------------------------------------------------- */
/* LM head fused with the display statistics (no reference counterpart:   */
/* the reference's statistics take materialised logits, csrc/ops.cpp:446). */
/* ---------------------------------------------------------------------- */

/* Workspace bytes cid_lm_head_display_statistics needs for rows x vocab. */
CID_API size_t cid_lm_head_workspace_bytes(int64_t rows, int64_t vocab);

/* display_token_statistics(token_ids, logits) of logits = hidden @ weight^T
 * without writing the logits: hidden rows x hidden_dim bf16 and weight
 * vocab x hidden_dim bf16, both row-major with hidden_dim % 8 == 0 and
 * 16-byte aligned bases (workspace too), rows <= 2^31 - 129; f32
 * accumulation on the tcgen05 tensor cores,
 * each logit rounded to bf16 first when round_bf16 != 0 (the statistics of
 * a bf16 LM head's stored output).  token_ids rows int64; outputs as
 * cid_display_token_statistics.  workspace: device memory of at least
 * cid_lm_head_workspace_bytes(rows, vocab) bytes.  Waits inside the kernel
 * are bounded; one that runs out sets CID_STATUS_LM_HEAD_TIMEOUT. */
CID_API int cid_lm_head_display_statistics(const void* hidden, int64_t rows, int64_t hidden_dim,
                        const void* weight, int64_t vocab, const int64_t* token_ids,
                        int round_bf16, float* confidence, int64_t* predicted,
                        float* current_confidence, void* workspace,
                        size_t workspace_bytes, uint32_t* status, void* stream);

/* The shard record (cid_display_shard_records) of every row over the logits
 * hidden @ weight_shard^T, whose rows are the global columns [vocab_offset,
 * vocab_offset + vocab_shard) of total_vocab, without writing those logits:
 * the per-rank half of a vocabulary-parallel LM head (the records of all
 * ranks then go through cid_display_combine_records).  Operands, rounding
 * and workspace (cid_lm_head_workspace_bytes(rows, vocab_shard)) as
 * cid_lm_head_display_statistics; records: rows x 16 bytes of device memory. */
CID_API int cid_lm_head_shard_records(const void* hidden, int64_t rows, int64_t hidden_dim,
                        const void* weight_shard, int64_t vocab_shard, int64_t vocab_offset,
                        int64_t total_vocab, const int64_t* token_ids, int round_bf16,
                        cid_shard_record_t* records, void* workspace, size_t workspace_bytes,
                        uint32_t* status, void* stream);

/* ---------------------------------------------------------------------- */
/* Peer record exchange (no reference counterpart: the multi-GPU form of   */
/* the vocabulary-parallel statistics, csrc/ops.cpp:446-474 sharded).      */
/* ---------------------------------------------------------------------- */

/* Bytes of one rank's inbox for `world` ranks (<= 8) and up to rows_capacity
 * (<= 2^31 - 1) rows: records [2][world][rows_capacity] then a 256-byte tail
 * (flag words); 0 for arguments outside those ranges. */
CID_API size_t cid_peer_inbox_bytes(int world, int64_t rows_capacity);
/* cudaMalloc'd, zeroed inbox on the current device (set-up, not per step). */
CID_API int cid_peer_inbox_alloc(size_t bytes, void** inbox);
CID_API int cid_peer_inbox_free(void* inbox);
/* CUDA IPC handle of an inbox (64 bytes), and its mapping in another process
 * of the same node (peer access over NVLink); release unmaps it. */
CID_API int cid_peer_inbox_export(void* inbox, unsigned char handle[64]);
CID_API int cid_peer_inbox_import(const unsigned char handle[64], void** peer_inbox);
CID_API int cid_peer_inbox_release(void* peer_inbox);

/* The shard records of cid_display_shard_records, each stored by the
 * statistics kernel as it finishes the row into this rank's slot (of the
 * epoch's parity) of every inbox: its own and, over peer memory, the other
 * ranks' (inboxes: `world` 16-byte-aligned device pointers as this process
 * maps them, inboxes[rank] its own); then `epoch` published in this rank's
 * flag word of every inbox (system fence, then release) by a kernel that
 * starts after the statistics kernel has completed.  1 <= rows <=
 * rows_capacity; `epoch` increases by one per step on every rank. */
CID_API int cid_display_shard_records_to_peers(cid_dtype_t dtype, const void* logits,
                        int64_t row_stride, const int64_t* token_ids, int64_t rows,
                        int64_t shard_vocab, int64_t vocab_offset, int64_t total_vocab,
                        int rank, int world, void* const* inboxes, int64_t rows_capacity,
                        uint32_t epoch, uint32_t* status, void* stream);

/* Any per-row shard records of this rank (rows x 16 bytes on the device,
 * e.g. from cid_lm_head_shard_records) stored into this rank's slot of every
 * inbox, own included, then `epoch` published as by
 * cid_display_shard_records_to_peers. */
CID_API int cid_peer_push_records(const cid_shard_record_t* records, int64_t rows, int rank,
                        int world, void* const* inboxes, int64_t rows_capacity, uint32_t epoch,
                        void* stream);

/* cid_display_combine_records over this rank's inbox once every rank has
 * published `epoch` there; the wait is bounded by wait_seconds (at most 60),
 * after which the statistics are NaN (predicted 0) and
 * CID_STATUS_PEER_TIMEOUT is set.  A peer found two or more epochs ahead
 * (before or after the rows are read) sets CID_STATUS_PEER_OUT_OF_STEP.
 * While either bit is set in *status, the exchange is poisoned: every
 * combine writes NaN statistics without waiting, until the caller clears the
 * word and builds a new exchange (fresh inboxes, epochs from 1). */
CID_API int cid_display_combine_inbox(void* inbox, int world, const int64_t* shard_offsets_host,
                        const int64_t* token_ids, int64_t rows, int64_t rows_capacity,
                        uint32_t epoch, double wait_seconds, float* confidence,
                        int64_t* predicted, float* current_confidence, uint32_t* status,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CID_ENGINE_B200_H */
