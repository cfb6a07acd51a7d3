// Migration copy kernel (see migrate.cu).
#pragma once
#include "common.cuh"

namespace dual {

struct MigrateParams {
  const int64_t* local_planes;   // [planes] device pointers of the local pool planes
  const int64_t* remote_planes;  // [banks * planes] device pointers of supplier planes (bank-major)
  int planes;                    // 72 = 36 layers x (K, V)
  int banks;                     // number of supplier banks (striping g % banks)
  const int64_t* source;         // [n] local slots (forward) / global remote ids (reverse)
  const int64_t* target;         // [n] global remote ids (forward) / local slots (reverse)
  int64_t n;
  int reverse;
  int64_t row_bytes;             // bytes per (slot, plane); multiple of 16
  int64_t local_slots;           // rows in every local plane
  int64_t remote_slots;          // rows in every supplier plane
  unsigned* status;
};

cudaError_t launch_migrate_copy(const MigrateParams& p, int max_ctas, cudaStream_t stream);

}  // namespace dual
