// Tiered causal append / prefill attention (tcgen05), see prefill.cu.
#pragma once
#include "decode.cuh"

namespace dual {

struct AppendParams {
  const __nv_bfloat16* q;  // [sum q, 32, 128]
  int64_t q_stride_tok, q_stride_head;
  const char* k_local;
  const char* v_local;
  int64_t local_stride;
  int64_t local_capacity;
  const char* peer_k[kMaxPeers];
  const char* peer_v[kMaxPeers];
  int num_peers;
  int64_t peer_stride;
  int64_t peer_slots;
  const int32_t* qo_indptr;  // [B+1]
  const int32_t* kv_indptr;  // [B+1]
  const int32_t* indices;    // unified page ids: history (any order) then the query suffix in order
  int64_t num_indices;
  int batch;
  int causal;
  float scale_log2;
  const int4* work;          // {request, kv head, query tile, cost} from append_plan
  int num_work;
  __nv_bfloat16* out;        // [sum q, 32, 128]
  int64_t out_stride_tok, out_stride_head;
  float* lse;                // [sum q, 32] base 2, or nullptr
  unsigned* status;
  uint32_t inject;           // DUAL_INJECT_* bits (tests only; 0 in production)
};

// Host-side schedule: one item {request, kv head, 64-token query pair, kv tiles} per pair, grouped by
// (request, kv head), groups longest first and pairs longest first within a group; with per-request
// remote counts (`remote`, may be null), the items of mostly-remote requests spread over the launch.
// Returns the number of items; writes min(n, max_work) items of 4 int32 into `work` (may be null).
int64_t append_plan(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* remote, int batch, int causal,
                    int32_t* work, int64_t max_work);
cudaError_t launch_tiered_append(const AppendParams& p, cudaStream_t stream);

}  // namespace dual
