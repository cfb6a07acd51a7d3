// Page-table kernels (see pack.cu).
#pragma once
#include "common.cuh"

namespace dual {

enum : unsigned { kStatusBadTier = 1u << 5 };

struct PackParams {
  int32_t* tier;            // [req_pool, stride]  (written only for the fused decode-step token)
  int32_t* slot;            // [req_pool, stride]
  int64_t rows;             // rows of both tables
  int64_t stride;           // row stride of both tables (elements) = max logical length
  const int32_t* req;       // [B] request-pool rows
  const int32_t* seq;       // [B] logical lengths
  const int32_t* prefix;    // [B] fully visible prefix lengths, or nullptr (= seq: decode)
  const int64_t* new_loc;   // [B] optional: local slot of the newest token (decode step)
  int batch;
  int64_t local_capacity;   // C; remote pages are encoded slot + C + 1
  int remote_rows;          // RN (0 = no interleave)
  int tile_rows;            // TN
  int32_t* full;            // sum(seq) entries
  int32_t* history;         // sum(prefix) entries or nullptr
  unsigned* status;         // optional
};

struct LayoutParams {
  int32_t* tier;
  int32_t* slot;
  int64_t rows;
  int64_t stride;
  const int32_t* req;       // [B]
  const int32_t* start;     // [B] offset of each request's locations, or nullptr (= b)
  const int32_t* length;    // [B] tokens to write, or nullptr (= 1)
  const int32_t* prefix;    // [B] first logical position written
  const int64_t* loc64;     // locations (int64), or
  const int32_t* loc32;     // locations (int32)
  int batch;
  unsigned* status;         // optional
};

cudaError_t launch_pack_read_order(const PackParams& p, cudaStream_t stream);
cudaError_t launch_write_layout(const LayoutParams& p, int max_len, cudaStream_t stream);

}  // namespace dual
