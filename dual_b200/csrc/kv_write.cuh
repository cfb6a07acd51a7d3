// New tokens' K/V rows into the local pool (see kv_write.cu).
#pragma once
#include "common.cuh"
#include "decode.cuh"

namespace dual {

struct KvWriteParams {
  char* k_local;              // local K / V pools of one layer: [C + 1] rows of 8 kv heads x 128 bf16
  char* v_local;
  int64_t local_stride;       // bytes between slots
  int64_t capacity;           // C: valid slots are 0 (SGLang's dummy) .. C
  const char* k;              // new rows, heads x dims contiguous, token stride in bytes
  const char* v;
  int64_t k_stride;
  int64_t v_stride;
  const int64_t* loc64;       // SGLang out_cache_loc (int64) or int32 locations
  const int32_t* loc32;
  int64_t n;
  unsigned* status;
};

cudaError_t launch_set_kv_buffer(const KvWriteParams& p, cudaStream_t stream);

}  // namespace dual
