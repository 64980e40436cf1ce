/* Known-answer tests through the C ABI only (no torch): the reference's
 * C++ KATs (tests/cpp/test_ops.cpp:10-64 of fwerkor/cid-engine v1.1.0), the
 * first-tie argmax KAT (tests/test_cuda.py:94-100), the same row through a
 * one-rank peer record exchange, and the fused LM head on exactly
 * representable logits.  Device memory comes from the CUDA runtime; every
 * entry point runs on the legacy default stream.  Exit status 0 = all passed. */
#include <cuda_runtime_api.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "cid_engine_b200.h"

#define CHECK(cond, msg)                       \
  do {                                         \
    if (!(cond)) {                             \
      fprintf(stderr, "FAILED: %s\n", msg);    \
      return 1;                                \
    }                                          \
  } while (0)

/* float32 statistics: within a pure relative 1e-5 of the exact value */
static int rel_close(float got, double expect) {
  return fabs((double)got - expect) <= 1e-5 * fabs(expect);
}

static void* dev_copy(const void* host, size_t bytes) {
  void* d = NULL;
  if (cudaMalloc(&d, bytes) != cudaSuccess) return NULL;
  cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
  return d;
}

int main(void) {
  /* prefix allocation: occupancy [1,4,1] {1,0,0,0}, logits {10,10,10,-10},
   * threshold 0.5, 2 allocations -> {0,1,1,0} (test_ops.cpp:10-29) */
  float occ[4] = {1, 0, 0, 0}, lg[4] = {10, 10, 10, -10};
  float* d_occ = dev_copy(occ, sizeof(occ));
  float* d_lg = dev_copy(lg, sizeof(lg));
  uint8_t* d_out = dev_copy((uint8_t[4]){9, 9, 9, 9}, 4);
  CHECK(d_occ && d_lg && d_out, "cudaMalloc");
  CHECK(cid_prefix_allocation_mask(CID_DTYPE_F32, d_occ, 4, 1, CID_DTYPE_F32, d_lg, 4, 1, 1, 4,
                                   0.5, 2, d_out, NULL) == CID_OK, "prefix launch");
  uint8_t sel[4];
  cudaMemcpy(sel, d_out, 4, cudaMemcpyDeviceToHost);
  CHECK(sel[0] == 0 && sel[1] == 1 && sel[2] == 1 && sel[3] == 0, "prefix allocation mismatch");

  /* linear assignment: costs [1,4,4], 3 active rows -> {1,0,2,-1}
   * (test_ops.cpp:33-53) */
  float costs[16] = {4, 1, 3, 8, 2, 0, 5, 7, 3, 2, 2, 6, 9, 9, 9, 9};
  int64_t counts[1] = {3};
  float* d_costs = dev_copy(costs, sizeof(costs));
  int64_t* d_counts = dev_copy(counts, sizeof(counts));
  int64_t* d_assign = dev_copy((int64_t[4]){7, 7, 7, 7}, 4 * sizeof(int64_t));
  CHECK(cid_batched_linear_assignment(CID_DTYPE_F32, d_costs, d_counts, 1, 4, 4, d_assign, NULL,
                                      NULL) == CID_OK, "assignment launch");
  int64_t assign[4];
  cudaMemcpy(assign, d_assign, sizeof(assign), cudaMemcpyDeviceToHost);
  CHECK(assign[0] == 1 && assign[1] == 0 && assign[2] == 2 && assign[3] == -1,
        "batched linear assignment mismatch");

  /* retired occupancy: lifecycle[0,1,2] = 1 retires slot 1 (test_ops.cpp:55-64) */
  float life[12] = {0};
  life[1 * 3 + 2] = 1.0f;
  float* d_life = dev_copy(life, sizeof(life));
  float* d_live = dev_copy(occ, sizeof(occ));
  CHECK(cid_live_slot_occupancy(CID_DTYPE_F32, d_occ, d_life, 4, 3, 2, d_live, NULL) == CID_OK,
        "live launch");
  float live[4];
  cudaMemcpy(live, d_live, sizeof(live), cudaMemcpyDeviceToHost);
  CHECK(live[1] == 0.0f && live[0] == 1.0f, "retired occupancy mismatch");

  /* statistics: logits {1,5,5,2}, id 2 -> argmax 1 (first of the tie),
   * confidence = current = e^0 / (e^-4 + 2 + e^-3) */
  float row[4] = {1, 5, 5, 2};
  int64_t id[1] = {2};
  float* d_row = dev_copy(row, sizeof(row));
  int64_t* d_id = dev_copy(id, sizeof(id));
  float* d_conf = dev_copy((float[1]){0}, 4);
  float* d_cur = dev_copy((float[1]){0}, 4);
  int64_t* d_pred = dev_copy((int64_t[1]){-5}, 8);
  CHECK(cid_display_token_statistics(CID_DTYPE_F32, d_row, 4, d_id, 1, 4, d_conf, d_pred, d_cur,
                                     NULL, NULL) == CID_OK, "stats launch");
  float conf, cur;
  int64_t pred;
  cudaMemcpy(&conf, d_conf, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&cur, d_cur, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&pred, d_pred, 8, cudaMemcpyDeviceToHost);
  const double expect = 1.0 / (exp(-4.0) + 2.0 + exp(-3.0));
  CHECK(pred == 1, "argmax must keep the first tie");
  CHECK(rel_close(conf, expect) && rel_close(cur, expect), "statistics mismatch");

  /* the same row through a one-rank peer exchange: inbox, records, combine */
  size_t inbox_bytes = cid_peer_inbox_bytes(1, 1);
  void* inbox = NULL;
  CHECK(inbox_bytes > 0 && cid_peer_inbox_alloc(inbox_bytes, &inbox) == CID_OK, "inbox alloc");
  void* inboxes[1] = {inbox};
  CHECK(cid_display_shard_records_to_peers(CID_DTYPE_F32, d_row, 4, d_id, 1, 4, 0, 4, 0, 1,
                                           inboxes, 1, 1u, NULL, NULL) == CID_OK,
        "records to peers launch");
  int64_t offs[2] = {0, 4};
  CHECK(cid_display_combine_inbox(inbox, 1, offs, d_id, 1, 1, 1u, 5.0, d_conf, d_pred, d_cur,
                                  NULL, NULL) == CID_OK, "combine inbox launch");
  cudaMemcpy(&conf, d_conf, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&cur, d_cur, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&pred, d_pred, 8, cudaMemcpyDeviceToHost);
  CHECK(pred == 1 && rel_close(conf, expect) && rel_close(cur, expect),
        "peer exchange statistics mismatch");
  CHECK(cid_peer_inbox_free(inbox) == CID_OK, "inbox free");

  /* LM head fused with the statistics: hidden = e_0 (bf16 1.0), weight column
   * 0 holds the logits exactly: 3 at columns 5 and 270 (a tie across vocabulary
   * tiles: the lower column wins), 1 at column 7 (the token), 0 elsewhere;
   * S = 2 + e^-2 + 297 e^-3 relative to the maximum */
  enum { H = 64, V = 300 };
  static uint16_t hid[H], wgt[V * H];
  hid[0] = 0x3F80;           /* 1.0 */
  wgt[5 * H] = 0x4040;       /* 3.0 */
  wgt[270 * H] = 0x4040;     /* 3.0 */
  wgt[7 * H] = 0x3F80;       /* 1.0 */
  int64_t lid[1] = {7};
  void* d_hid = dev_copy(hid, sizeof(hid));
  void* d_wgt = dev_copy(wgt, sizeof(wgt));
  int64_t* d_lid = dev_copy(lid, sizeof(lid));
  size_t ws_bytes = cid_lm_head_workspace_bytes(1, V);
  void* d_ws = NULL;
  CHECK(d_hid && d_wgt && d_lid && cudaMalloc(&d_ws, ws_bytes) == cudaSuccess, "cudaMalloc");
  CHECK(cid_lm_head_display_statistics(d_hid, 1, H, d_wgt, V, d_lid, 1, d_conf, d_pred, d_cur,
                                       d_ws, ws_bytes, NULL, NULL) == CID_OK, "lm head launch");
  cudaMemcpy(&conf, d_conf, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&cur, d_cur, 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(&pred, d_pred, 8, cudaMemcpyDeviceToHost);
  const double s_lm = 2.0 + exp(-2.0) + 297.0 * exp(-3.0);
  CHECK(pred == 5, "lm head argmax must keep the first tie");
  CHECK(rel_close(conf, 1.0 / s_lm) && rel_close(cur, exp(-2.0) / s_lm),
        "lm head statistics mismatch");

  CHECK(cudaDeviceSynchronize() == cudaSuccess, "device error");
  printf("cid-engine B200 C-ABI known-answer tests passed\n");
  return 0;
}
