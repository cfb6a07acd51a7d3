// Tiered split-KV paged GQA decode for sm_100a.
//
// Replaces the FlashInfer FA2 batch-prefill JIT module that the reference
// patches with `paged_kv_t::tiered_address` and uses for decode
// (final/cooperative_4gpu/code/peer/flashinfer_peer.py:27-78 resolver,
// :105-142 module, hook peer/backend.py:132-138).  Page ids follow the same
// encoding: p <= C is local slot p; p > C is global remote id g = p - C - 1,
// held by supplier bank g % num_peers at physical slot g / num_peers
// (peer/flashinfer_peer.py:44-54, peer/remote_bank.py:1,21).
//
// Design (B200-first, page_size 1):
//   * One CTA (one per SM) owns a contiguous range of the flattened token
//     axis [g*T/G, (g+1)*T/G) for all 8 kv heads.  The range may span several
//     requests; each request-segment is flushed as one partial state.
//   * A producer warp stages the range's page ids into shared memory with
//     cp.async well ahead of use, resolves each page id once, and issues ONE
//     cp.async.bulk per token row and plane (2 KiB, contiguous in the NHD
//     pool), local HBM and peer HBM alike (no multicast), into an NS-deep
//     shared-memory ring completed by mbarrier transaction counts.
//   * 8 consumer warps, one per kv head, compute every tile with bf16
//     m16n8k16 tensor-core MMAs (the 4 query heads of the GQA group are the
//     MMA rows) and an exp2-domain online softmax.
//   * A request that lies inside one CTA's range is normalised in registers
//     and written directly.  A request split across CTAs leaves one partial
//     (O, m, d) state per CTA in the workspace; the last warp to finish a
//     (request, kv head) -- found with a per-(request, kv head) arrival
//     counter -- combines them with a log-sum-exp reduction and writes the
//     bf16 output and the base-2 LSE (FlashInfer's convention), then resets
//     the counter for the next launch.  No second kernel.
#pragma once
#include "common.cuh"

namespace dual {

constexpr int kHeadDim = 128;
constexpr int kNumQoHeads = 32;
constexpr int kNumKvHeads = 8;
constexpr int kGqa = kNumQoHeads / kNumKvHeads;  // 4 query heads per kv head
constexpr int kMaxPeers = 8;
constexpr int kPartialStride = 132;  // floats per (segment, q head): O[128], m, d, pad

struct TieredDecodeParams {
  const __nv_bfloat16* q;  // [B, 32, 128]
  int64_t q_stride_tok, q_stride_head;  // elements
  const char* k_local;     // local pool, page p at k_local + p * local_stride (bytes)
  const char* v_local;
  int64_t local_stride;    // bytes per slot (heads contiguous, 256 B each)
  int64_t local_capacity;  // C: valid local pages are 0..C
  const char* peer_k[kMaxPeers];
  const char* peer_v[kMaxPeers];
  int num_peers;
  int64_t peer_stride;     // bytes per slot in every supplier bank
  int64_t peer_slots;      // physical slots per supplier bank
  const int32_t* indptr;   // [B+1]
  const int32_t* indices;  // unified page ids, indptr[B] entries
  int64_t num_indices;     // capacity of `indices` (reads never go beyond it)
  int batch;
  float scale_log2;        // sm_scale * log2(e)
  float* partial;          // workspace: partial states
  unsigned* counters;      // workspace: arrival counter per (request, kv head), zero between launches
  unsigned* status;        // workspace status word
  int grid_g;              // CTAs per head group
  __nv_bfloat16* out;      // [B, 32, 128]
  int64_t out_stride_tok, out_stride_head;
  float* lse;              // [B, 32] (base 2) or nullptr
};

// One CTA = all 8 kv heads of a token range, so every token row of a plane is
// one contiguous 2 KiB block moved by ONE bulk copy (the TMA engine sustains
// HBM rate only for copies of ~2 KiB; 512 B copies cap near 3 TB/s).
template <int NS_, int TILE_>
struct DecodeConfig {
  static constexpr int NS = NS_;        // ring stages
  static constexpr int TILE = TILE_;    // token rows per stage
  static constexpr int ROW_BYTES = kNumKvHeads * kHeadDim * 2;  // 2048 B per token per plane
  static constexpr int PITCH = ROW_BYTES + 16;                  // +16 B: conflict-free ldmatrix rows
  static constexpr int PLANE_BYTES = TILE * PITCH;
  static constexpr int STAGE_BYTES = 2 * PLANE_BYTES;
  static constexpr int CONSUMERS = kNumKvHeads;                 // one warp per kv head
  static constexpr int THREADS = (CONSUMERS + 1) * 32;
  static constexpr int IDX_CHUNK = 512;                         // page ids staged per chunk
  static constexpr int IDX_BUFS = 3;
  static constexpr int SMEM_BYTES = NS * STAGE_BYTES + IDX_BUFS * IDX_CHUNK * 4 + (2 * NS + IDX_BUFS) * 8 + 16;
  static constexpr int ROWS = kNumQoHeads;                      // q heads per CTA
  static_assert(TILE == 16, "consumer MMA tiling assumes 16 token rows per stage");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

using DecodeCfg = DecodeConfig<3, 16>;

// Workspace layout: [status: 256 B][counters: batch x 8 kv heads x 4 B, rounded up to 256 B]
//                   [partials: (G + B) segments x 32 q heads x 132 floats].
inline size_t decode_counter_bytes(int batch) {
  return (size_t(batch) * kNumKvHeads * sizeof(unsigned) + 255) / 256 * 256;
}
inline size_t decode_workspace_head_bytes(int batch) { return 256 + decode_counter_bytes(batch); }
inline size_t decode_workspace_bytes(int batch, int grid_g) {
  return decode_workspace_head_bytes(batch) + sizeof(float) * size_t(grid_g + batch) * DecodeCfg::ROWS * kPartialStride;
}

cudaError_t launch_tiered_decode(const TieredDecodeParams& p, cudaStream_t stream);
int decode_default_grid_g(int device);

}  // namespace dual
