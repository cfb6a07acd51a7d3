// Tiered split-KV paged decode kernel + partial-state merge (see decode.cuh).
#include "decode.cuh"

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
    int l = 0, r = batch - 1;  // first request whose end exceeds lo
    while (l < r) {
      const int mid = (l + r) >> 1;
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

__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

constexpr float kDecodeRescale = 8.0f;  // log2 units

// Split of the flattened token axis [0, T) over G CTAs: CTA g owns [g T / G, (g + 1) T / G).
struct Split {
  int64_t T;
  int G;
  __device__ __forceinline__ int owner(int64_t x) const { return int(((x + 1) * G - 1) / T); }
  __device__ __forceinline__ bool nonempty(int g) const { return (int64_t(g) * T) / G < (int64_t(g + 1) * T) / G; }
  // [start, end) of request b, clamped into [0, T]
  __device__ __forceinline__ void range(const int32_t* indptr, int b, int64_t& start, int64_t& end) const {
    start = __ldg(indptr + b);
    end = __ldg(indptr + b + 1);
    start = start < 0 ? 0 : (start > T ? T : start);
    end = end < start ? start : (end > T ? T : end);
  }
};

// Combine the partial states of request b for the 4 q heads of kv head h (one warp) and write the
// bf16 output and the base-2 LSE.  CTAs glo..ghi cover the request; those with an empty range
// wrote nothing.  Partials are read through L2 (other SMs wrote them during this launch).  The loads
// of all four heads of a segment are independent and issued together, two segments at a time, so a
// merge costs a few L2 round trips rather than one per value.
__device__ __noinline__ void merge_request_heads(const TieredDecodeParams& p, const Split& sp, int b, int h,
                                                 int glo, int ghi, int lane) {
  constexpr int64_t kSeg = int64_t(kNumQoHeads) * kPartialStride;
  const float* base = p.partial + (int64_t(b) * kNumQoHeads + h * kGqa) * kPartialStride;
  float M[kGqa];
#pragma unroll
  for (int r = 0; r < kGqa; ++r) M[r] = -INFINITY;
#pragma unroll 4
  for (int gg = glo; gg <= ghi; ++gg) {
    if (!sp.nonempty(gg)) continue;
#pragma unroll
    for (int r = 0; r < kGqa; ++r) M[r] = fmaxf(M[r], __ldcg(base + gg * kSeg + r * kPartialStride + kHeadDim));
  }
  float D[kGqa];
  float4 acc[kGqa];
#pragma unroll
  for (int r = 0; r < kGqa; ++r) {
    D[r] = 0.f;
    acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll 2
  for (int gg = glo; gg <= ghi; ++gg) {
    if (!sp.nonempty(gg)) continue;
    float2 md[kGqa];
    float4 v[kGqa];
#pragma unroll
    for (int r = 0; r < kGqa; ++r) {
      const float* src = base + gg * kSeg + r * kPartialStride;
      md[r] = __ldcg(reinterpret_cast<const float2*>(src + kHeadDim));
      v[r] = __ldcg(reinterpret_cast<const float4*>(src) + lane);
    }
#pragma unroll
    for (int r = 0; r < kGqa; ++r) {
      const float w = (md[r].x == -INFINITY) ? 0.f : exp2f(md[r].x - M[r]);
      D[r] += w * md[r].y;
      acc[r].x += w * v[r].x;
      acc[r].y += w * v[r].y;
      acc[r].z += w * v[r].z;
      acc[r].w += w * v[r].w;
    }
  }
#pragma unroll
  for (int r = 0; r < kGqa; ++r) {
    const int row = h * kGqa + r;
    const float inv = 1.f / D[r];
    __nv_bfloat16* orow = p.out + int64_t(b) * p.out_stride_tok + int64_t(row) * p.out_stride_head;
    reinterpret_cast<__nv_bfloat162*>(orow + lane * 4)[0] = __floats2bfloat162_rn(acc[r].x * inv, acc[r].y * inv);
    reinterpret_cast<__nv_bfloat162*>(orow + lane * 4)[1] = __floats2bfloat162_rn(acc[r].z * inv, acc[r].w * inv);
    if (p.lse != nullptr && lane == 0) p.lse[int64_t(b) * kNumQoHeads + row] = M[r] + log2f(D[r]);
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1) tiered_decode_kernel(const __grid_constant__ TieredDecodeParams p) {
  constexpr int NS = Cfg::NS, TILE = Cfg::TILE, CONS = Cfg::CONSUMERS;
  constexpr int IC = Cfg::IDX_CHUNK, IB = Cfg::IDX_BUFS;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  int32_t* sidx = reinterpret_cast<int32_t*>(smem + NS * Cfg::STAGE_BYTES);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sidx + IB * IC);
  uint64_t* empty_bar = full_bar + NS;
  uint64_t* idx_bar = empty_bar + NS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(idx_bar + IB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;
  const int G = p.grid_g;

  // Zero the ring once so rows past the end of a partial tile are finite.
  {
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < NS * Cfg::STAGE_BYTES / 16; i += blockDim.x) reinterpret_cast<uint4*>(ring)[i] = z;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, CONS);
    }
    for (int s = 0; s < IB; ++s) mbar_init(idx_bar + s, 32);
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
  const Split sp{T, G};

  if (warp == CONS) {
    // ------------------------------------------------------------ producer
    TileIter<TILE> it;
    it.init(lo, hi, p.indptr, p.batch);
    const int r = lane & 15;
    const bool is_v = lane >= 16;
    const char* local_base = is_v ? p.v_local : p.k_local;
    const uint64_t policy = l2_policy_evict_first();
    const int64_t nchunks = (hi - lo + IC - 1) / IC;
    int64_t issued = 0, ready = -1;
    auto issue_chunk = [&](int64_t c) {
      const int buf = int(c % IB);
      const int64_t base = lo + c * IC;
      for (int i = lane; i < IC; i += 32)
        if (base + i < hi) cp_async_4(sidx + buf * IC + i, p.indices + base + i);
      cp_async_mbar_arrive_noinc(idx_bar + buf);
    };
    while (issued < nchunks && issued < IB) issue_chunk(issued++);
    int n_issued = 0;
    for (; it.valid(); it.next(p.indptr, p.batch), ++n_issued) {
      const int rows = it.rows();
      const int64_t c_first = (it.t0 - lo) / IC, c_last = (it.t0 + rows - 1 - lo) / IC;
      while (issued < nchunks && issued <= c_first + IB - 1) issue_chunk(issued++);
      bool ok = !*abort_flag;
      while (ok && ready < c_last) {
        ++ready;
        ok = mbar_wait_bounded(idx_bar + (ready % IB), uint32_t(ready / IB) & 1u);
      }
      const int stage = n_issued % NS;
      const int fill = n_issued / NS;
      if (ok && fill > 0) ok = mbar_wait_bounded(empty_bar + stage, (fill - 1) & 1);
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.status, kStatusWaitTimeout);
        break;
      }
      if (lane == 0) mbar_arrive_expect_tx(full_bar + stage, uint32_t(rows) * 2u * Cfg::ROW_BYTES);
      __syncwarp();
      if (r < rows) {
        const int64_t off = it.t0 + r - lo;
        const uint32_t page = static_cast<uint32_t>(sidx[int((off / IC) % IB) * IC + int(off % IC)]);
        const char* src;
        if (page <= static_cast<uint64_t>(p.local_capacity)) {
          src = local_base + int64_t(page) * p.local_stride;
        } else {
          const uint32_t gid = page - static_cast<uint32_t>(p.local_capacity) - 1u;
          const int np = p.num_peers;
          const uint32_t bank = np > 0 ? gid % uint32_t(np) : 0u;
          const uint32_t phys = np > 0 ? gid / uint32_t(np) : 0u;
          if (np <= 0 || int64_t(phys) >= p.peer_slots) {
            atomicOr(p.status, kStatusBadRemoteSlot);
            src = local_base;  // page 0 (SGLang's dummy slot): finite, in bounds
          } else {
            src = (is_v ? p.peer_v[bank] : p.peer_k[bank]) + int64_t(phys) * p.peer_stride;
          }
        }
        unsigned char* dst = ring + stage * Cfg::STAGE_BYTES + (is_v ? Cfg::PLANE_BYTES : 0) + r * Cfg::PITCH;
        bulk_g2s_hint(dst, src, Cfg::ROW_BYTES, full_bar + stage, policy);
      }
    }
    // Never leave the CTA with copies still landing in shared memory.
    asm volatile("cp.async.wait_all;" ::: "memory");
    const int outstanding = n_issued < NS ? n_issued : NS;
    for (int k = 0; k < outstanding; ++k) {
      const int n = n_issued - 1 - k;
      if (!mbar_wait_bounded(full_bar + (n % NS), (n / NS) & 1)) {
        atomicOr(p.status, kStatusWaitTimeout);
        break;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int h = warp;  // kv head
  const int gi = lane >> 2, ci = lane & 3;

  TileIter<TILE> it;
  it.init(lo, hi, p.indptr, p.batch);

  uint32_t qa[8][2];
  float o[16][4];
  float m_run = -INFINITY, d_run = 0.f;
  int cur_b = -1;
  int n_seen = 0;
  constexpr int kDeferredMerges = 4;
  int deferred[kDeferredMerges];  // requests this warp merges once its range is done
  int n_deferred = 0;

  auto load_q = [&](int b) {
    if (gi < kGqa) {
      const __nv_bfloat16* qrow = p.q + int64_t(b) * p.q_stride_tok + int64_t(h * kGqa + gi) * p.q_stride_head;
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
    }
    const int stage = n_seen % NS;
    const int fill = n_seen / NS;
    const int rows = it.rows();
    bool ok = !*abort_flag;
    if (ok && !mbar_wait_bounded(full_bar + stage, fill & 1)) {
      *abort_flag = 1;
      atomicOr(p.status, kStatusWaitTimeout);
      ok = false;
    }
    if (ok) {
      const unsigned char* sK = ring + stage * Cfg::STAGE_BYTES + h * kHeadDim * 2;
      const unsigned char* sV = sK + Cfg::PLANE_BYTES;
      const int mi = lane >> 3, rr = lane & 7;
      // ---- S = Q K^T  (rows: 4 q heads, cols: 16 tokens)
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kp = 0; kp < 4; ++kp) {
          uint32_t b0, b1, b2, b3;
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
      // Lazy rescaling: the reference point m_run moves (and O, d are rescaled) only when the tile
      // max exceeds it by more than 2^kDecodeRescale, so P <= 256 in between; the partial state
      // (O, m, d) stays exact because O and d share the reference point.  Rescaling every tile
      // was 64 multiplies per lane per 16 tokens.
      float alpha = 1.f;
      if (tmax > m_run + kDecodeRescale) {
        alpha = fast_exp2(m_run - tmax);  // 0 on a segment's first tile
        m_run = tmax;
      }
      float pr[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) pr[e] = fast_exp2(x[e] - m_run);
      d_run = d_run * alpha + (pr[0] + pr[1]) + (pr[2] + pr[3]);
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
          o[nt][0] *= alpha;
          o[nt][1] *= alpha;
          o[nt][2] *= alpha;
          o[nt][3] *= alpha;
        }
      }
      // P as a hi + lo pair of bf16 values, keeping P's bf16 rounding out of the output: hi feeds
      // MMA rows g (the 4 query heads), lo feeds the otherwise idle rows g + 8 of the same MMA;
      // the two accumulator halves are added when the segment is flushed.
      uint32_t pa0, pa2, pl0, pl2;
      split_bf16x2(pr[0], pr[1], pa0, pl0);
      split_bf16x2(pr[2], pr[3], pa2, pl2);
      // ---- O += P V
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3, sV + ((mi & 1) * 8 + rr) * Cfg::PITCH + (dp * 16 + (mi >> 1) * 8) * 2);
        mma_bf16_16816(o[2 * dp], pa0, pl0, pa2, pl2, b0, b1);
        mma_bf16_16816(o[2 * dp + 1], pa0, pl0, pa2, pl2, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar + stage);
    if (it.last_in_segment()) {
      float d_row = d_run;
      d_row += __shfl_xor_sync(0xffffffffu, d_row, 1);
      d_row += __shfl_xor_sync(0xffffffffu, d_row, 2);
      int64_t start, end;
      sp.range(p.indptr, cur_b, start, end);
      const bool whole = start >= lo && end <= hi;  // the request lies inside this CTA's range
      if (gi < kGqa) {
        if (whole) {
          // ---- normalise and write the output directly
          const float inv = 1.f / d_row;
          __nv_bfloat16* orow =
              p.out + int64_t(cur_b) * p.out_stride_tok + int64_t(h * kGqa + gi) * p.out_stride_head;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt)
            *reinterpret_cast<__nv_bfloat162*>(orow + nt * 8 + 2 * ci) =
                __floats2bfloat162_rn((o[nt][0] + o[nt][2]) * inv, (o[nt][1] + o[nt][3]) * inv);
          if (ci == 0 && p.lse != nullptr) p.lse[int64_t(cur_b) * kNumQoHeads + h * kGqa + gi] = m_run + log2f(d_row);
        } else {
          // ---- one partial state (unnormalised O, m, d) of a request split across CTAs
          float* dst = p.partial + (int64_t(g + cur_b) * Cfg::ROWS + h * kGqa + gi) * kPartialStride;
#pragma unroll
          for (int nt = 0; nt < 16; ++nt)
            *reinterpret_cast<float2*>(dst + nt * 8 + 2 * ci) = make_float2(o[nt][0] + o[nt][2], o[nt][1] + o[nt][3]);
          if (ci == 0) *reinterpret_cast<float2*>(dst + kHeadDim) = make_float2(m_run, d_row);
        }
      }
      reset_state();
      if (!whole) {
        // the last of the request's CTAs to arrive for this kv head merges the partial states
        __syncwarp();
        const int glo = sp.owner(start), ghi = sp.owner(end - 1);
        int segments = 0;
        for (int gg = glo; gg <= ghi; ++gg) segments += sp.nonempty(gg) ? 1 : 0;
        unsigned last = 0;
        if (lane == 0) {
          __threadfence();  // this warp's partial is visible before its arrival is counted
          unsigned* cnt = p.counters + int64_t(cur_b) * kNumKvHeads + h;
          last = atomicAdd(cnt, 1u) == unsigned(segments - 1) ? 1u : 0u;
          if (last) *cnt = 0u;  // every arrival of this launch is in: ready for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          // merge after this warp's range is done (a merge in mid-stream would hold up the CTA's
          // pipeline); only when the short list is full is it done at once
          if (n_deferred < kDeferredMerges) {
            deferred[n_deferred++] = cur_b;
          } else {
            __threadfence();
            merge_request_heads(p, sp, cur_b, h, glo, ghi, lane);
          }
        }
      }
    }
  }

  // ---- the merges this warp deferred (it was the last of their CTAs to arrive)
  if (n_deferred > 0) __threadfence();
  for (int i = 0; i < n_deferred; ++i) {
    int64_t start, end;
    sp.range(p.indptr, deferred[i], start, end);
    merge_request_heads(p, sp, deferred[i], h, sp.owner(start), sp.owner(end - 1), lane);
  }

  // ---- requests with no KV entries: output 0, LSE -inf, written by the CTA that owns their
  // position in the token axis (the last CTA for positions at the end; CTA 0 when T = 0)
  for (int b = lane; b < p.batch; b += 32) {
    int64_t start, end;
    sp.range(p.indptr, b, start, end);
    if (end > start) continue;
    const int own = T == 0 ? 0 : (start < T ? sp.owner(start) : G - 1);
    if (own != g) continue;
    for (int r = 0; r < kGqa; ++r) {
      const int row = h * kGqa + r;
      __nv_bfloat16* orow = p.out + int64_t(b) * p.out_stride_tok + int64_t(row) * p.out_stride_head;
      for (int d = 0; d < kHeadDim; d += 2)
        *reinterpret_cast<__nv_bfloat162*>(orow + d) = __floats2bfloat162_rn(0.f, 0.f);
      if (p.lse != nullptr) p.lse[int64_t(b) * kNumQoHeads + row] = -INFINITY;
    }
  }
}

}  // namespace

int decode_default_grid_g(int device) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms < 1 ? 1 : sms;
}

cudaError_t launch_tiered_decode(const TieredDecodeParams& p, cudaStream_t stream) {
  using Cfg = DecodeCfg;
  static std::atomic<uint64_t> configured{0};
  if (cudaError_t e = set_max_dynamic_smem_once(tiered_decode_kernel<Cfg>, Cfg::SMEM_BYTES, configured))
    return e;
  tiered_decode_kernel<Cfg><<<p.grid_g, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
