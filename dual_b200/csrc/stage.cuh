// Per-layer staging of supplier rows into local memory (see stage.cu).
#pragma once
#include "common.cuh"
#include "decode.cuh"

namespace dual {

struct StageParams {
  const char* peer_k[kMaxPeers];  // supplier bank planes of one layer (K, V), [bank_slots] rows each
  const char* peer_v[kMaxPeers];
  char* stage_k[kMaxPeers];       // local stage buffers, same row numbering as the banks
  char* stage_v[kMaxPeers];
  int banks;
  int64_t peer_stride;            // bytes between rows of a bank plane
  int64_t stage_stride;           // bytes between rows of a stage buffer
  int64_t bank_slots;             // rows per bank (and per stage buffer)
  int64_t row_bytes;              // bytes copied per row (2048 = 8 kv heads x 128 x bf16); multiple of 16
  const int32_t* indices;         // unified index list of the forward
  int64_t n;
  int64_t local_capacity;         // C: entries > C are remote
  unsigned* status;
};

// One warp per CTA, one CTA per 32 index entries by default: many small CTAs spread the copy over
// every SM.  The copy is issued before the attention, not beside it: measured on config-4 shapes,
// issuing it beside a running tiered_append_kernel made the pair ~1 ms slower than copy + append
// back to back (a copy CTA cannot share an SM with an append CTA, whose 11 warps x 160 registers
// leave too few, so copy CTAs only take SMs from the append).
constexpr int kStageThreads = 32;

cudaError_t launch_stage_rows(const StageParams& p, int max_ctas, cudaStream_t stream);

}  // namespace dual
