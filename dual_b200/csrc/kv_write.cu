// The KV writer in front of tiered attention: new tokens' K and V rows into their local slots.
//
// Replaces SGLang's MHATokenToKVPool.set_kv_buffer as the reference calls it before every
// tiered attention launch (final/vendor/nvlink_prefill_timing/.../backend.py:34,42): the
// positions a forward creates are always local (tier 0), so row i of k / v goes to slot loc[i] of
// the layer's K / V pool.  Bit-exact byte copy.
//
// B200 shape: a warp moves one token -- K and V rows of 2 KiB each, 4 + 4 16-byte loads per lane
// issued before any store -- and walks tokens grid-stride.  A slot outside [0, C] is skipped and
// recorded in the status word (slot 0 is SGLang's dummy slot, which padded batch entries write).
#include "kv_write.cuh"

namespace dual {
namespace {

constexpr int kWriteThreads = 256;
constexpr int kRowBytes = kNumKvHeads * kHeadDim * 2;  // 2048
constexpr int kChunks = kRowBytes / 16 / 32;           // 16-byte chunks per lane per row: 4

__device__ __forceinline__ uint4 ld_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(kWriteThreads) set_kv_buffer_kernel(const __grid_constant__ KvWriteParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = int64_t(gridDim.x) * (kWriteThreads / 32);
  for (int64_t i = int64_t(blockIdx.x) * (kWriteThreads / 32) + (threadIdx.x >> 5); i < p.n; i += warps_total) {
    const int64_t slot = p.loc64 ? p.loc64[i] : int64_t(p.loc32[i]);
    if (slot < 0 || slot > p.capacity) {
      if (lane == 0) atomicOr(p.status, kStatusBadLocalSlot);
      continue;
    }
    const char* ks = p.k + i * p.k_stride;
    const char* vs = p.v + i * p.v_stride;
    char* kd = p.k_local + slot * p.local_stride;
    char* vd = p.v_local + slot * p.local_stride;
    uint4 a[kChunks], b[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      a[c] = ld_v4(ks + (c * 32 + lane) * 16);
      b[c] = ld_v4(vs + (c * 32 + lane) * 16);
    }
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      st_v4(kd + (c * 32 + lane) * 16, a[c]);
      st_v4(vd + (c * 32 + lane) * 16, b[c]);
    }
  }
}

}  // namespace

cudaError_t launch_set_kv_buffer(const KvWriteParams& p, cudaStream_t stream) {
  if (p.n <= 0) return cudaSuccess;
  constexpr int64_t kPerCta = kWriteThreads / 32;
  int64_t ctas = (p.n + kPerCta - 1) / kPerCta;
  if (ctas > 4 * 148) ctas = 4 * 148;
  set_kv_buffer_kernel<<<int(ctas), kWriteThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
