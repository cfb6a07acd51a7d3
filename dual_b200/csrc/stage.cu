// Per-layer staging of the supplier rows one forward reads.
//
// Restates LayerStager.launch (final/cooperative_4gpu/code/peer/staging.py:27-38).  The reference
// copies each supplier bank's whole layer into a local one-layer buffer before that layer's
// prefill reads it (prefill_backend.py:33), so the attention kernel sees remote rows at local
// cost.  Here only the rows the index list references move: entry p > C is global remote id
// g = p - C - 1 -> bank g % n, row g / n, and both planes (K, V) of that row are copied to the
// same row of the bank's local stage buffer.  The stage buffers then stand in for the banks in
// the attention call with the index list unchanged.
//
// Why the append path wants it: the append kernel reads every history row once per 64-token
// query pair of its request, and this GPU's L2 does not cache a peer's memory, so without
// staging every re-read crosses NVLink; staged, each remote row crosses once per layer.
//
// Shape: a warp loads 32 index entries, ballots the remote ones and copies them two entries at
// a time -- K and V rows of both, row_bytes / 512 16-byte non-coherent loads per lane per row in
// flight -- then stores them.
#include "stage.cuh"

namespace dual {
namespace {

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Streaming store (evict-first in L2): the staged rows are read by the next launch, once per query
// pair, and that launch's own reuse should keep L2.
__device__ __forceinline__ void st_cs_v4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Source and destination of the K and V rows of global remote id g; false (status recorded by
// lane 0) when the row is beyond the bank.
__device__ __forceinline__ bool resolve(const StageParams& p, int64_t g, int lane, const char* src[2],
                                        char* dst[2]) {
  const int64_t bank = g % p.banks;
  const int64_t row = g / p.banks;
  if (row >= p.bank_slots) {
    if (lane == 0) atomicOr(p.status, kStatusBadRemoteSlot);
    return false;
  }
  src[0] = p.peer_k[bank] + row * p.peer_stride;
  src[1] = p.peer_v[bank] + row * p.peer_stride;
  dst[0] = p.stage_k[bank] + row * p.stage_stride;
  dst[1] = p.stage_v[bank] + row * p.stage_stride;
  return true;
}

__global__ void __launch_bounds__(kStageThreads) stage_rows_kernel(const __grid_constant__ StageParams p) {
  constexpr int kWarps = kStageThreads / 32;
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = int64_t(gridDim.x) * kWarps;
  const int64_t warp_id = int64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  const int chunks = int(p.row_bytes / 16);
  for (int64_t base = warp_id * 32; base < p.n; base += warps_total * 32) {
    const int64_t i = base + lane;
    int64_t g = -1;
    if (i < p.n) {
      const int64_t e = p.indices[i];
      if (e > p.local_capacity) g = e - p.local_capacity - 1;
    }
    unsigned remote = __ballot_sync(0xffffffffu, g >= 0);
    while (remote != 0u) {
      const int l0 = __ffs(remote) - 1;
      remote &= remote - 1u;
      const int l1 = remote != 0u ? __ffs(remote) - 1 : -1;
      if (l1 >= 0) remote &= remote - 1u;
      const int64_t g0 = __shfl_sync(0xffffffffu, g, l0);
      const int64_t g1 = __shfl_sync(0xffffffffu, g, l1 >= 0 ? l1 : l0);
      const char* src[4];
      char* dst[4];
      bool ok[4];
      ok[0] = ok[1] = resolve(p, g0, lane, src, dst);
      ok[2] = ok[3] = l1 >= 0 && resolve(p, g1, lane, src + 2, dst + 2);
      for (int c = lane; c < chunks; c += 32 * 4) {
        uint4 v[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int cc = c + 32 * k;
            if (ok[r] && cc < chunks) v[r][k] = ld_nc_v4(src[r] + int64_t(cc) * 16);
          }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int cc = c + 32 * k;
            if (ok[r] && cc < chunks) st_cs_v4(dst[r] + int64_t(cc) * 16, v[r][k]);
          }
      }
    }
  }
}

}  // namespace

cudaError_t launch_stage_rows(const StageParams& p, int max_ctas, cudaStream_t stream) {
  if (p.n <= 0) return cudaSuccess;
  const int64_t per_cta = int64_t(kStageThreads / 32) * 32;
  int64_t ctas = (p.n + per_cta - 1) / per_cta;
  if (max_ctas > 0 && ctas > max_ctas) ctas = max_ctas;
  stage_rows_kernel<<<int(ctas), kStageThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
