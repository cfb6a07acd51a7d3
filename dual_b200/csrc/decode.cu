// Tiered split-KV paged decode kernel + partial-state merge (see decode.cuh).
#include "decode.cuh"

#include <cfloat>

namespace dual {
namespace {

// Walks the tiles of one CTA's token range [lo, hi): tiles never straddle a
// request boundary, so each request segment ends with a (possibly partial) tile.
template <int TILE>
struct TileIter {
  int64_t t0, seg_hi, hi;
  int b;
  __device__ __forceinline__ void init(int64_t lo, int64_t hi_, const int32_t* indptr, int batch) {
    hi = hi_;
    t0 = lo;
    b = 0;
    seg_hi = hi;
    if (lo >= hi) return;
    // first request whose end exceeds lo
    int l = 0, r = batch - 1;
    while (l < r) {
      int mid = (l + r) >> 1;
      if (int64_t(__ldg(indptr + mid + 1)) > lo) r = mid; else l = mid + 1;
    }
    b = l;
    seg_hi = min(hi, int64_t(__ldg(indptr + b + 1)));
  }
  __device__ __forceinline__ bool valid() const { return t0 < hi; }
  __device__ __forceinline__ int rows() const { return int(min(int64_t(TILE), seg_hi - t0)); }
  __device__ __forceinline__ bool last_in_segment() const { return t0 + TILE >= seg_hi; }
  __device__ __forceinline__ void next(const int32_t* indptr, int batch) {
    t0 += rows();
    if (t0 >= seg_hi && t0 < hi) {
      do {
        if (b + 1 >= batch) {  // only reachable with a non-monotone indptr: stop, never read past it
          t0 = hi;
          return;
        }
        ++b;
        seg_hi = min(hi, int64_t(__ldg(indptr + b + 1)));
      } while (seg_hi <= t0);
    }
  }
};

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1) tiered_decode_kernel(const __grid_constant__ TieredDecodeParams p) {
  constexpr int HG = Cfg::HG, NS = Cfg::NS, TILE = Cfg::TILE, NPH = Cfg::NPH;
  constexpr int CONS = Cfg::CONSUMERS;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  float* red = reinterpret_cast<float*>(smem + NS * Cfg::STAGE_BYTES);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + NS * Cfg::STAGE_BYTES + Cfg::RED_FLOATS * 4);
  uint64_t* empty_bar = full_bar + NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty_bar + NS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hg = blockIdx.x % Cfg::NHG;
  const int g = blockIdx.x / Cfg::NHG;
  const int G = p.grid_g;

  // Zero the ring once so rows past the end of a partial tile are finite.
  {
    uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < NS * Cfg::STAGE_BYTES / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(ring)[i] = z;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, HG);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  fence_proxy_async_smem();
  __syncthreads();

  int64_t T = __ldg(p.indptr + p.batch);
  if (T > p.num_indices || T < 0) {
    if (threadIdx.x == 0) atomicOr(p.status, kStatusBadLength);
    T = T < 0 ? 0 : p.num_indices;
  }
  const int64_t lo = (int64_t(g) * T) / G;
  const int64_t hi = (int64_t(g + 1) * T) / G;

  if (warp == CONS) {
    // ------------------------------------------------------------ producer
    TileIter<TILE> it, pf;
    it.init(lo, hi, p.indptr, p.batch);
    pf = it;
    const int r = lane & 15;
    const bool is_v = lane >= 16;
    const char* local_base = is_v ? p.v_local : p.k_local;
    const int64_t head_off = int64_t(hg) * Cfg::ROW_BYTES;
    const uint64_t policy = l2_policy_evict_first();
    // index prefetch: 4 tiles ahead, one index per lane (row r)
    int32_t q0 = 0, q1 = 0, q2 = 0, q3 = 0;
    auto fetch = [&](TileIter<TILE>& t) -> int32_t {
      int32_t v = 0;
      if (t.valid()) {
        if (r < t.rows()) v = __ldg(p.indices + t.t0 + r);
        t.next(p.indptr, p.batch);
      }
      return v;
    };
    q0 = fetch(pf);
    q1 = fetch(pf);
    q2 = fetch(pf);
    q3 = fetch(pf);
    int n_issued = 0;
    bool aborted = false;
    for (; it.valid(); it.next(p.indptr, p.batch), ++n_issued) {
      const int32_t page_id = q0;
      q0 = q1;
      q1 = q2;
      q2 = q3;
      q3 = fetch(pf);
      const int stage = n_issued % NS;
      const int fill = n_issued / NS;
      if (fill > 0) {
        if (*abort_flag || !mbar_wait_bounded(empty_bar + stage, (fill - 1) & 1)) {
          *abort_flag = 1;
          atomicOr(p.status, kStatusWaitTimeout);
          aborted = true;
          break;
        }
      }
      const int rows = it.rows();
      if (lane == 0) mbar_arrive_expect_tx(full_bar + stage, uint32_t(rows) * 2u * Cfg::ROW_BYTES);
      __syncwarp();
      if (r < rows) {
        const uint32_t page = static_cast<uint32_t>(page_id);
        const char* src;
        if (page <= static_cast<uint64_t>(p.local_capacity)) {
          src = local_base + int64_t(page) * p.local_stride + head_off;
        } else {
          const uint32_t gid = page - static_cast<uint32_t>(p.local_capacity) - 1u;
          const int np = p.num_peers;
          if (np <= 0) {
            atomicOr(p.status, kStatusBadRemoteSlot);
            src = local_base + head_off;
          } else {
            const uint32_t bank = gid % uint32_t(np);
            const uint32_t phys = gid / uint32_t(np);
            if (int64_t(phys) >= p.peer_slots) {
              atomicOr(p.status, kStatusBadRemoteSlot);
              src = local_base + head_off;
            } else {
              src = (is_v ? p.peer_v[bank] : p.peer_k[bank]) + int64_t(phys) * p.peer_stride + head_off;
            }
          }
        }
        unsigned char* dst = ring + stage * Cfg::STAGE_BYTES + (is_v ? Cfg::PLANE_BYTES : 0) + r * Cfg::PITCH;
        bulk_g2s_hint(dst, src, Cfg::ROW_BYTES, full_bar + stage, policy);
      }
    }
    // Never leave the CTA with bulk copies still landing in shared memory.
    const int outstanding = n_issued < NS ? n_issued : NS;
    for (int k = 0; k < outstanding; ++k) {
      const int n = n_issued - 1 - k;
      if (!mbar_wait_bounded(full_bar + (n % NS), (n / NS) & 1)) {
        atomicOr(p.status, kStatusWaitTimeout);
        break;
      }
    }
    (void)aborted;
    return;
  }

  // -------------------------------------------------------------- consumers
  const int h = warp % HG;   // kv head within the group
  const int ph = warp / HG;  // tile phase
  const int gi = lane >> 2, ci = lane & 3;
  const int kvh = hg * HG + h;
  const int nconsumer_threads = CONS * 32;

  TileIter<TILE> it;
  it.init(lo, hi, p.indptr, p.batch);

  uint32_t qa[8][2];
  float o[16][4];
  float m_run = -INFINITY, d_run = 0.f;
  int cur_b = -1;
  int j = 0;  // tile index within the current segment
  int n_seen = 0;

  auto load_q = [&](int b) {
    if (gi < kGqa) {
      const __nv_bfloat16* qrow = p.q + int64_t(b) * p.q_stride_tok + int64_t(kvh * kGqa + gi) * p.q_stride_head;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * ci);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * ci);
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) qa[ks][0] = qa[ks][1] = 0u;
    }
  };
  auto reset_state = [&]() {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    m_run = -INFINITY;
    d_run = 0.f;
  };
  reset_state();

  for (; it.valid(); it.next(p.indptr, p.batch), ++n_seen) {
    if (it.b != cur_b) {
      cur_b = it.b;
      load_q(cur_b);
      j = 0;
    }
    const int stage = n_seen % NS;
    const int fill = n_seen / NS;
    const int rows = it.rows();
    if ((j % NPH) == ph) {
      bool ok = !*abort_flag;
      if (ok && !mbar_wait_bounded(full_bar + stage, fill & 1)) {
        *abort_flag = 1;
        atomicOr(p.status, kStatusWaitTimeout);
        ok = false;
      }
      if (ok) {
        const unsigned char* sK = ring + stage * Cfg::STAGE_BYTES + h * kHeadDim * 2;
        const unsigned char* sV = sK + Cfg::PLANE_BYTES;
        // ---- S = Q K^T  (rows: 4 q heads, cols: 16 tokens)
        float s[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
          for (int kp = 0; kp < 4; ++kp) {
            uint32_t b0, b1, b2, b3;
            const int mi = lane >> 3, rr = lane & 7;
            ldmatrix_x4(b0, b1, b2, b3, sK + (nt * 8 + rr) * Cfg::PITCH + (kp * 32 + mi * 8) * 2);
            mma_bf16_16816(s[nt], qa[2 * kp][0], 0u, qa[2 * kp][1], 0u, b0, b1);
            mma_bf16_16816(s[nt], qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u, b2, b3);
          }
        }
        // ---- online softmax in the exp2 domain
        float x[4];
        x[0] = s[0][0] * p.scale_log2;
        x[1] = s[0][1] * p.scale_log2;
        x[2] = s[1][0] * p.scale_log2;
        x[3] = s[1][1] * p.scale_log2;
        if (rows < TILE) {
          const int t0 = 2 * ci;
          if (t0 >= rows) x[0] = -INFINITY;
          if (t0 + 1 >= rows) x[1] = -INFINITY;
          if (8 + t0 >= rows) x[2] = -INFINITY;
          if (8 + t0 + 1 >= rows) x[3] = -INFINITY;
        }
        float tmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float m_new = fmaxf(m_run, tmax);
        const float alpha = fast_exp2(m_run - m_new);
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = fast_exp2(x[e] - m_new);
        d_run = d_run * alpha + (pr[0] + pr[1]) + (pr[2] + pr[3]);
        m_run = m_new;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          o[nt][0] *= alpha;
          o[nt][1] *= alpha;
        }
        const uint32_t pa0 = pack_bf16x2(pr[0], pr[1]);
        const uint32_t pa2 = pack_bf16x2(pr[2], pr[3]);
        // ---- O += P V
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int mi = lane >> 3, rr = lane & 7;
          ldmatrix_x4_trans(b0, b1, b2, b3, sV + ((mi & 1) * 8 + rr) * Cfg::PITCH + (dp * 16 + (mi >> 1) * 8) * 2);
          mma_bf16_16816(o[2 * dp], pa0, 0u, pa2, 0u, b0, b1);
          mma_bf16_16816(o[2 * dp + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar + stage);
    }
    ++j;
    if (it.last_in_segment()) {
      // ---- flush this request segment: merge the NPH phase states per head
      float d_row = d_run;
      d_row += __shfl_xor_sync(0xffffffffu, d_row, 1);
      d_row += __shfl_xor_sync(0xffffffffu, d_row, 2);
      if (gi < kGqa) {
        float* dst = red + ((ph * HG + h) * kGqa + gi) * kPartialStride;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          dst[nt * 8 + 2 * ci] = o[nt][0];
          dst[nt * 8 + 2 * ci + 1] = o[nt][1];
        }
        if (ci == 0) {
          dst[kHeadDim] = m_run;
          dst[kHeadDim + 1] = d_row;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nconsumer_threads) : "memory");
      const int64_t slot = int64_t(hg) * (G + p.batch) + g + cur_b;
      float* gdst = p.partial + slot * Cfg::ROWS * kPartialStride;
      for (int idx = threadIdx.x; idx < Cfg::ROWS * (kHeadDim + 2); idx += nconsumer_threads) {
        const int row = idx / (kHeadDim + 2), col = idx % (kHeadDim + 2);
        const int hh = row / kGqa, qq = row % kGqa;
        float M = -INFINITY;
#pragma unroll
        for (int q = 0; q < NPH; ++q) M = fmaxf(M, red[((q * HG + hh) * kGqa + qq) * kPartialStride + kHeadDim]);
        float acc = 0.f;
        if (col == kHeadDim) {
          acc = M;
        } else {
#pragma unroll
          for (int q = 0; q < NPH; ++q) {
            const float* src = red + ((q * HG + hh) * kGqa + qq) * kPartialStride;
            const float w = (src[kHeadDim] == -INFINITY) ? 0.f : fast_exp2(src[kHeadDim] - M);
            acc += w * (col == kHeadDim + 1 ? src[kHeadDim + 1] : src[col]);
          }
        }
        gdst[row * kPartialStride + col] = acc;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nconsumer_threads) : "memory");
      reset_state();
    }
  }
}

// Combine the partial states of each (request, q head) and write the output.
template <class Cfg>
__global__ void __launch_bounds__(Cfg::ROWS * 32) decode_merge_kernel(const __grid_constant__ TieredDecodeParams p) {
  const int b = blockIdx.x;
  const int hg = blockIdx.y;
  const int row = threadIdx.x >> 5;  // 0..7 : q head within the head group
  const int lane = threadIdx.x & 31;
  const int G = p.grid_g;
  int64_t T = __ldg(p.indptr + p.batch);
  if (T > p.num_indices || T < 0) T = T < 0 ? 0 : p.num_indices;
  int64_t start = __ldg(p.indptr + b), end = __ldg(p.indptr + b + 1);
  start = start < 0 ? 0 : (start > T ? T : start);
  end = end < start ? start : (end > T ? T : end);
  const int qh = hg * Cfg::ROWS + row;
  __nv_bfloat16* orow = p.out + int64_t(b) * p.out_stride_tok + int64_t(qh) * p.out_stride_head;
  if (end <= start || T <= 0) {
    for (int d = lane; d < kHeadDim; d += 32) orow[d] = __float2bfloat16(0.f);
    if (p.lse != nullptr && lane == 0) p.lse[int64_t(b) * kNumQoHeads + qh] = -INFINITY;
    return;
  }
  auto gof = [&](int64_t x) -> int { return int(((x + 1) * G - 1) / T); };
  const int glo = gof(start), ghi = gof(end - 1);
  const float* base = p.partial + (int64_t(hg) * (G + p.batch) + b) * Cfg::ROWS * kPartialStride +
                      row * kPartialStride;
  // CTAs with an empty range (T < G) wrote no partial state: skip them.
  auto nonempty = [&](int gg) { return (int64_t(gg) * T) / G < (int64_t(gg + 1) * T) / G; };
  float M = -INFINITY;
  for (int gg = glo; gg <= ghi; ++gg)
    if (nonempty(gg)) M = fmaxf(M, base[int64_t(gg) * Cfg::ROWS * kPartialStride + kHeadDim]);
  float D = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int gg = glo; gg <= ghi; ++gg) {
    if (!nonempty(gg)) continue;
    const float* src = base + int64_t(gg) * Cfg::ROWS * kPartialStride;
    const float mm = src[kHeadDim];
    const float w = (mm == -INFINITY) ? 0.f : exp2f(mm - M);
    D += w * src[kHeadDim + 1];
    const float4 v = *reinterpret_cast<const float4*>(src + lane * 4);
    acc[0] += w * v.x;
    acc[1] += w * v.y;
    acc[2] += w * v.z;
    acc[3] += w * v.w;
  }
  const float inv = 1.f / D;
  __nv_bfloat162 o01 = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
  __nv_bfloat162 o23 = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  reinterpret_cast<__nv_bfloat162*>(orow + lane * 4)[0] = o01;
  reinterpret_cast<__nv_bfloat162*>(orow + lane * 4)[1] = o23;
  if (p.lse != nullptr && lane == 0) p.lse[int64_t(b) * kNumQoHeads + qh] = M + log2f(D);
}

}  // namespace

int decode_default_grid_g(int device) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int g = sms / DecodeCfg::NHG;
  return g < 1 ? 1 : g;
}

cudaError_t launch_tiered_decode(const TieredDecodeParams& p, cudaStream_t stream) {
  using Cfg = DecodeCfg;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tiered_decode_kernel<Cfg>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  tiered_decode_kernel<Cfg><<<p.grid_g * Cfg::NHG, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.batch > 0) {
    decode_merge_kernel<Cfg><<<dim3(p.batch, Cfg::NHG), Cfg::ROWS * 32, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  return e;
}

}  // namespace dual
