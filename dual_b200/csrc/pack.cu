// Page-table kernels: read-order packer and new-token layout writer.
//
// pack_read_order restates, as one CUDA kernel per forward:
//   * decode: Triton `_count_remote` + `_pack_indices`
//     (final/cooperative_4gpu/code/peer/backend.py:22-79), which the reference
//     audits against `history_order(encoded, far, length, RN, TN)`
//     (peer/backend.py:95-103, peer/layout.py:5-22);
//   * prefill/append: Triton `packing.prepare` (peer/packing.py:6-36), stable
//     tier compaction + RN-remote / (TN-RN)-local interleave of the fully
//     visible prefix, query suffix left in place, `Full` and `History` lists.
// Decode is the prefill case with prefix == length.  Unlike the reference
// decode packer, arbitrary tier maps are handled (not only a remote prefix);
// on remote-prefix maps both produce the same list.
//
// write_layout restates Triton `_write_prefill_layout` (peer/page_ops.py:6-18)
// and the per-step decode slot/tier write (V/nvlink_short_serving/backend.py:100-101).
#include "pack.cuh"

namespace dual {
namespace {

constexpr int kPackThreads = 512;
constexpr int kPackItems = 8;
constexpr int kPackChunk = kPackThreads * kPackItems;

// Block-wide exclusive scan of a packed (far << 32 | near) counter.
__device__ __forceinline__ uint64_t block_exclusive_scan(uint64_t v, uint64_t* warp_tot, uint64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    constexpr int NW = kPackThreads / 32;
    uint64_t t = lane < NW ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint64_t y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < NW) warp_tot[lane] = t;  // inclusive warp prefix
  }
  __syncthreads();
  total = warp_tot[kPackThreads / 32 - 1];
  const uint64_t before = warp == 0 ? 0 : warp_tot[warp - 1];
  __syncthreads();  // warp_tot reused by the next call
  return before + x - v;
}

__global__ void __launch_bounds__(kPackThreads) pack_read_order_kernel(const __grid_constant__ PackParams p) {
  __shared__ uint64_t warp_tot[kPackThreads / 32];
  __shared__ long long s_start[2];
  __shared__ int s_count;
  const int b = blockIdx.x;
  const int rid = p.req[b];
  const int n = p.seq[b];
  const int pfx = p.prefix ? p.prefix[b] : n;
  const bool row_ok = rid >= 0 && rid < p.rows && n >= 0 && n <= p.stride && pfx >= 0 && pfx <= n;
  int32_t* tier_row = p.tier + int64_t(row_ok ? rid : 0) * p.stride;
  int32_t* slot_row = p.slot + int64_t(row_ok ? rid : 0) * p.stride;

  // Output offsets: exclusive prefix sums of lengths / prefixes over requests.
  {
    long long a = 0, c = 0;
    for (int i = threadIdx.x; i < b; i += blockDim.x) {
      a += p.seq[i];
      c += p.prefix ? p.prefix[i] : p.seq[i];
    }
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    if (threadIdx.x == 0) { s_start[0] = 0; s_start[1] = 0; s_count = 0; }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&s_start[0]), static_cast<unsigned long long>(a));
      atomicAdd(reinterpret_cast<unsigned long long*>(&s_start[1]), static_cast<unsigned long long>(c));
    }
  }
  // Optional fused decode-step write of the newest token (always local).
  if (row_ok && p.new_loc != nullptr && threadIdx.x == 0 && n > 0) {
    slot_row[n - 1] = static_cast<int32_t>(p.new_loc[b]);
    tier_row[n - 1] = 0;
  }
  if (!row_ok) {
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusBadLength);
    return;
  }
  __syncthreads();
  const long long full_start = s_start[0], hist_start = s_start[1];

  const int RN = p.remote_rows, TN = p.tile_rows;
  const uint32_t enc_off = static_cast<uint32_t>(p.local_capacity) + 1u;

  // pass 1: remote count among the prefix
  int r = 0;
  if (RN > 0) {
    int cnt = 0;
    for (int i = threadIdx.x; i < pfx; i += blockDim.x) cnt += (tier_row[i] == 1);
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s_count, cnt);
    __syncthreads();
    r = s_count;
  }
  const int l = pfx - r;
  const int LN = TN - RN;
  int groups = 0, base = 0, tail_r = 0, tail_l = 0, tail_size = 0;
  if (RN > 0) {
    groups = min(r / RN, l / LN);
    base = groups * TN;
    const int rleft = r - groups * RN, lleft = l - groups * LN;
    tail_r = min(rleft, RN);
    tail_l = min(lleft, LN);
    const int extra_l = min(TN - tail_r - tail_l, lleft - tail_l);
    tail_l += extra_l;
    tail_r += min(TN - tail_r - tail_l, rleft - tail_r);
    tail_size = tail_r + tail_l;
  }

  // pass 2: ranks, destinations, writes
  uint64_t carry = 0;
  for (int c0 = 0; c0 < n; c0 += kPackChunk) {
    const int p0 = c0 + threadIdx.x * kPackItems;
    int32_t tv[kPackItems], sv[kPackItems];
    uint64_t mine = 0;
#pragma unroll
    for (int k = 0; k < kPackItems; ++k) {
      const int pos = p0 + k;
      tv[k] = 0;
      sv[k] = 0;
      if (pos < n) {
        tv[k] = tier_row[pos];
        sv[k] = slot_row[pos];
        if (pos < pfx) mine += (tv[k] == 1) ? (uint64_t(1) << 32) : uint64_t(1);
      }
    }
    uint64_t total;
    uint64_t excl = block_exclusive_scan(mine, warp_tot, total) + carry;
    carry += total;
    int rr = int(excl >> 32), ll = int(excl & 0xffffffffu);
#pragma unroll
    for (int k = 0; k < kPackItems; ++k) {
      const int pos = p0 + k;
      if (pos >= n) break;
      const bool far = tv[k] == 1;
      const int32_t encoded = static_cast<int32_t>(static_cast<uint32_t>(sv[k]) + (far ? enc_off : 0u));
      int dest = pos;
      if (pos < pfx) {
        if (RN > 0) {
          if (far) {
            dest = rr < groups * RN ? (rr / RN) * TN + rr % RN
                 : rr < groups * RN + tail_r ? base + rr - groups * RN
                 : base + tail_size + rr - groups * RN - tail_r;
            ++rr;
          } else {
            dest = ll < groups * LN ? (ll / LN) * TN + RN + ll % LN
                 : ll < groups * LN + tail_l ? base + tail_r + ll - groups * LN
                 : base + tail_size + ll - groups * LN - tail_l;
            ++ll;
          }
        }
        if (p.history) p.history[hist_start + dest] = encoded;
        if (p.status && tv[k] != 0 && tv[k] != 1) atomicOr(p.status, kStatusBadTier);
      }
      p.full[full_start + dest] = encoded;
    }
  }
}

__global__ void write_layout_kernel(const __grid_constant__ LayoutParams p) {
  const int b = blockIdx.x;
  const int off = blockIdx.y * blockDim.x + threadIdx.x;
  const int len = p.length ? p.length[b] : 1;
  if (off >= len) return;
  const int rid = p.req[b];
  const int pfx = p.prefix[b];
  if (rid < 0 || rid >= p.rows || pfx < 0 || int64_t(pfx) + len > p.stride) {
    if (off == 0 && p.status) atomicOr(p.status, kStatusBadLength);
    return;
  }
  const int64_t start = p.start ? p.start[b] : b;
  const int64_t loc = p.loc64 ? p.loc64[start + off] : int64_t(p.loc32[start + off]);
  const int64_t idx = int64_t(rid) * p.stride + pfx + off;
  p.slot[idx] = static_cast<int32_t>(loc);
  p.tier[idx] = 0;
}

}  // namespace

cudaError_t launch_pack_read_order(const PackParams& p, cudaStream_t stream) {
  if (p.batch <= 0) return cudaSuccess;
  pack_read_order_kernel<<<p.batch, kPackThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_write_layout(const LayoutParams& p, int max_len, cudaStream_t stream) {
  if (p.batch <= 0 || max_len <= 0) return cudaSuccess;
  dim3 grid(p.batch, (max_len + 255) / 256);
  write_layout_kernel<<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
