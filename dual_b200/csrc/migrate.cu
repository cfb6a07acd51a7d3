// Token-slot migration copy: N slots x all (layer, K|V) planes in one launch.
//
// Restates the reference's Triton `_copy` (final/cooperative_4gpu/code/peer/fused_copy.py:6-33):
// local slot s <-> global remote id g, supplier bank g % banks, physical slot
// g / banks, for every plane (36 layers x K,V = 72 in the reference), byte-exact.
// forward (reverse == 0): local -> remote (P2P stores to the supplier);
// reverse  (reverse == 1): remote -> local (ratio repair / restore).
//
// B200 shape: each (slot, plane) row is one contiguous `row_bytes` block at
// both ends (2 KB for 8 kv heads x 128 x bf16).  A warp moves two rows per
// iteration with 16-byte non-coherent loads (8 in flight per lane) and plain
// 16-byte stores; the grid is kept small (a side-stream copy that competes
// with decode for SMs), and each CTA walks rows grid-stride.
#include "migrate.cuh"

namespace dual {
namespace {

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Resolve row `w` (token i = w / planes, plane pl = w % planes) to (src, dst);
// returns false (and records the error) if a slot is out of range.
__device__ __forceinline__ bool resolve_row(const MigrateParams& p, int64_t w, const char*& src, char*& dst) {
  const int64_t i = w / p.planes;
  const int pl = int(w % p.planes);
  const int64_t s = p.source[i];
  const int64_t t = p.target[i];
  const int64_t global_remote = p.reverse ? s : t;
  const int64_t local_slot = p.reverse ? t : s;
  if (local_slot < 0 || local_slot >= p.local_slots || global_remote < 0) {
    atomicOr(p.status, kStatusBadCopySlot);
    return false;
  }
  const int64_t bank = global_remote % p.banks;
  const int64_t phys = global_remote / p.banks;
  if (phys >= p.remote_slots) {
    atomicOr(p.status, kStatusBadCopySlot);
    return false;
  }
  char* lp = reinterpret_cast<char*>(p.local_planes[pl]) + local_slot * p.row_bytes;
  char* rp = reinterpret_cast<char*>(p.remote_planes[bank * p.planes + pl]) + phys * p.row_bytes;
  if (p.reverse) { src = rp; dst = lp; } else { src = lp; dst = rp; }
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) != 0u) {
    atomicOr(p.status, kStatusBadCopySlot);
    return false;
  }
  return true;
}

constexpr int kCopyThreads = 256;

// At most 64 registers a thread (16,384 per CTA), so one copy CTA fits on an SM beside a running
// decode CTA (288 threads x 168 registers = 48,384 of the SM's 65,536): a migration launched while
// decode holds every SM then runs alongside it instead of only in the gaps between layers.
__global__ void __launch_bounds__(kCopyThreads, 4) migrate_copy_kernel(const __grid_constant__ MigrateParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = int64_t(gridDim.x) * (kCopyThreads / 32);
  const int64_t warp_id = int64_t(blockIdx.x) * (kCopyThreads / 32) + (threadIdx.x >> 5);
  const int64_t rows = p.n * p.planes;
  const int chunks = int(p.row_bytes / 16);  // 16-byte chunks per row
  for (int64_t w0 = warp_id * 2; w0 < rows; w0 += warps_total * 2) {
    const char* src[2];
    char* dst[2];
    bool ok[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) ok[u] = (w0 + u < rows) && resolve_row(p, w0 + u, src[u], dst[u]);
    for (int c = lane; c < chunks; c += 32 * 4) {
      uint4 v[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int cc = c + 32 * k;
          if (ok[u] && cc < chunks) v[u][k] = ld_nc_v4(src[u] + int64_t(cc) * 16);
        }
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int cc = c + 32 * k;
          if (ok[u] && cc < chunks) st_v4(dst[u] + int64_t(cc) * 16, v[u][k]);
        }
    }
  }
}

}  // namespace

cudaError_t launch_migrate_copy(const MigrateParams& p, int max_ctas, cudaStream_t stream) {
  if (p.n <= 0) return cudaSuccess;
  const int64_t rows = p.n * p.planes;
  const int64_t rows_per_cta = (kCopyThreads / 32) * 2;
  int64_t ctas = (rows + rows_per_cta - 1) / rows_per_cta;
  if (max_ctas > 0 && ctas > max_ctas) ctas = max_ctas;
  migrate_copy_kernel<<<int(ctas), kCopyThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
