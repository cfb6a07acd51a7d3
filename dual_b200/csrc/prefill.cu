// Tiered causal append / prefill attention on the 5th-generation tensor cores (tcgen05).
//
// Replaces the reference's tiered FA2 batch-prefill module for the append path
// (final/cooperative_4gpu/code/peer/prefill_backend.py:25-42 run hook, JIT module
// peer/flashinfer_peer.py:105-142) and drops its per-layer staging of supplier
// banks into local HBM (peer/staging.py): remote rows are read in place by peer
// loads, local and remote alike.
//
// Semantics (FlashInfer paged prefill, page_size 1): request b has q_b query tokens
// (qo_indptr) and L_b kv entries (kv_indptr); with `causal`, query token i sees list
// entry j iff j < L_b - q_b (the fully visible, possibly re-ordered history) or
// j - (L_b - q_b) <= i (the query suffix, kept in order by the packer); without
// `causal` every entry is visible.  Output bf16 [sum q, 32, 128], LSE base 2.
//
// Design (one CTA per work item = request x kv head x 64 query tokens, warp-specialised):
//   * two query tiles of 32 tokens x 4 GQA heads = 2 x 128 MMA rows share every K/V tile;
//   * loader warps (2) gather 64-entry K/V tiles (256 B of this kv head per entry, local HBM
//     or a supplier's HBM through peer loads) with 16-byte cp.async, 16 lanes per entry so every
//     warp instruction moves whole cache lines, into a 5-stage ring of 128B-swizzled tiles; each
//     loader arrives on the stage's barrier when its copies land (cp.async.mbarrier.arrive), so
//     the loaders run up to the ring depth ahead of the tensor core;
//   * one MMA thread issues S_q = Q_q K^T (tcgen05.mma M128 N64 K16, fp32 in TMEM) for both
//     query tiles, then O_q += P_q V (M128 N128 K16) once the softmax of tile q is done, so
//     the tensor core runs QK of one query tile while the other is in softmax;
//   * one softmax warpgroup per query tile (thread = TMEM lane = row): mask only on tiles that
//     cross the causal diagonal or the end, scale + exp2 as one FMA + one MUFU per score,
//     lazy rescaling of O (the reference max moves only when it grows by more than 2^8),
//     P written to tensor memory (tcgen05.st) as a bf16 pair hi + lo (P's bf16 rounding would
//     otherwise move short-row outputs by ~4e-3 under cancellation) and consumed from there by
//     the PV MMA; epilogue O / rowsum -> bf16, LSE = m + log2 rowsum.
// All waits are bounded; a timed-out wait records DUAL_STATUS_WAIT_TIMEOUT and every role
// unwinds (no thread is left at a barrier the others skipped).
#include <algorithm>
#include <vector>

#include "decode.cuh"
#include "prefill.cuh"
#include "tcgen05.cuh"

namespace dual {
namespace {

constexpr int kQTok = 32;                  // query tokens per query tile
constexpr int kRows = kQTok * kGqa;        // 128 MMA rows per query tile
constexpr int kQTiles = 2;                 // query tiles per CTA
constexpr int kPairTok = kQTok * kQTiles;  // 64 query tokens per work item
constexpr int kBN = 64;                    // kv entries per kv tile
constexpr int kNS = 5;                     // kv ring stages
constexpr int kLoadWarps = 2;
constexpr int kLoadThreads = kLoadWarps * 32;
constexpr int kSoftmaxWarps = 4 * kQTiles;
constexpr int kMmaWarp = kSoftmaxWarps + kLoadWarps;  // warp 10
constexpr int kThreads = (kMmaWarp + 1) * 32;          // 352
constexpr float kRescaleThreshold = 8.0f;  // log2 units: p stays <= 256 between rescales

constexpr int kQBytes = kRows * 256;       // 32 KB: [128 rows x 128 dims] bf16
constexpr int kKVBytes = kBN * 256;        // 16 KB: [64 entries x 128 dims] bf16
// smem: Q0 Q1 | (K, V) x kNS stages | barriers   (P lives in tensor memory)
constexpr int kOffQ = 0;
constexpr int kOffKV = kQTiles * kQBytes;
constexpr int kOffBar = kOffKV + kNS * 2 * kKVBytes;
constexpr int kNumBars = 2 * kNS + 3 * kQTiles + 1;
constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

// TMEM columns: S0 [0,64) S1 [64,128) O0 [128,256) O1 [256,384)
//               P0 hi [384,416) lo [416,448)  P1 hi [448,480) lo [480,512)   (bf16 pairs per column)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColP = 384;

__device__ __forceinline__ void cp_async_16_zfill(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(kThreads, 1) tiered_append_kernel(const __grid_constant__ AppendParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;                      // [kNS]  count kLoadThreads
  uint64_t* kv_empty = bars + kNS;               // [kNS]  count 1 (tcgen05.commit)
  uint64_t* s_full = bars + 2 * kNS;             // [2]    count 1 (tcgen05.commit)
  uint64_t* p_full = s_full + kQTiles;           // [2]    count 128 (softmax warpgroup)
  uint64_t* o_done = p_full + kQTiles;           // [2]    count 1 (tcgen05.commit)
  uint64_t* q_full = o_done + kQTiles;           // [1]    count kLoadThreads
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kNumBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars) + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 w = p.work[blockIdx.x];
  const int b = w.x, h = w.y, pair = w.z;
  const int64_t q0 = p.qo_indptr[b], q_len = int64_t(p.qo_indptr[b + 1]) - q0;
  const int64_t kv0 = p.kv_indptr[b], L = int64_t(p.kv_indptr[b + 1]) - kv0;
  const int64_t t_begin = int64_t(pair) * kPairTok;
  const int64_t t_end = min(q_len, t_begin + kPairTok);
  const int64_t prefix = L - q_len;
  if (q_len <= 0 || t_begin >= q_len) return;
  if (L < 0 || (p.causal && prefix < 0) || kv0 < 0 || kv0 + L > p.num_indices) {
    if (tid == 0) atomicOr(p.status, kStatusBadLength);
    return;
  }
  const int64_t kv_end = p.causal ? min(L, prefix + t_end) : L;
  const int ntiles = int((kv_end + kBN - 1) / kBN);

  if (tid == 0) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(kv_full + s, kLoadThreads);
      mbar_init(kv_empty + s, 1);
    }
    for (int q = 0; q < kQTiles; ++q) {
      mbar_init(s_full + q, 1);
      mbar_init(p_full + q, kRows);
      mbar_init(o_done + q, 1);
    }
    mbar_init(q_full, kLoadThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tc::alloc(tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity)) return true;
    *abort_flag = 1;
    atomicOr(p.status, kStatusWaitTimeout);
    return false;
  };

  if (warp >= kSoftmaxWarps && warp < kMmaWarp) {
    // ================================================================ loaders
    const int lt = tid - kSoftmaxWarps * 32;  // 0..63
    // query tiles: 256 rows x 16 chunks of 16 B, 64 threads
    for (int i = lt; i < kQTiles * kRows; i += kLoadThreads) {
      const int q = i / kRows, r = i % kRows;
      const int64_t tok = t_begin + q * kQTok + r / kGqa;
      const bool valid = tok < t_end;
      const __nv_bfloat16* src =
          p.q + (q0 + (valid ? tok : 0)) * p.q_stride_tok + int64_t(h * kGqa + r % kGqa) * p.q_stride_head;
      unsigned char* dst = smem + kOffQ + q * kQBytes;
#pragma unroll
      for (int c = 0; c < 16; ++c) cp_async_16_zfill(dst + tc::sw128_offset<kRows>(r, c), src + c * 8, valid);
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async_smem();
    mbar_arrive(q_full);
    // kv tiles: loader warp lw owns entries [32 lw, 32 lw + 32) of each tile; lane l prefetches the
    // page id of entry 32 lw + l, then 16 lanes cover one entry's 256 B (two full 128 B lines) so each
    // warp-wide cp.async moves two entries, coalesced.
    const int lw = lt >> 5;
    const int half = lane >> 4, chunk = lane & 15;
    auto page_of = [&](int jj) -> int32_t {  // page id of entry 32 lw + lane of tile jj (0 past the end)
      const int64_t pos = int64_t(jj) * kBN + 32 * lw + lane;
      return pos < kv_end ? p.indices[kv0 + pos] : 0;
    };
    int32_t page_a = page_of(0), page_b = ntiles > 1 ? page_of(1) : 0;  // two tiles of look-ahead
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int s = j % kNS, f = j / kNS;
      const int32_t my_page = page_a;
      page_a = page_b;
      page_b = j + 2 < ntiles ? page_of(j + 2) : 0;
      if (f > 0 && !wait(kv_empty + s, (f - 1) & 1)) {
        ok = false;
        break;
      }
      const int64_t tile0 = int64_t(j) * kBN;
      unsigned char* sk = smem + kOffKV + s * 2 * kKVBytes;
      unsigned char* sv = sk + kKVBytes;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int row = 32 * lw + 2 * i + half;  // entry within the tile
        const uint32_t page = static_cast<uint32_t>(__shfl_sync(0xffffffffu, my_page, 2 * i + half));
        const bool valid = tile0 + row < kv_end;
        const char* ksrc = p.k_local;
        const char* vsrc = p.v_local;
        if (valid) {
          if (page <= static_cast<uint64_t>(p.local_capacity)) {
            ksrc = p.k_local + int64_t(page) * p.local_stride;
            vsrc = p.v_local + int64_t(page) * p.local_stride;
          } else {
            const uint32_t gid = page - static_cast<uint32_t>(p.local_capacity) - 1u;
            const int np = p.num_peers;
            const uint32_t bank = np > 0 ? gid % uint32_t(np) : 0u;
            const uint32_t phys = np > 0 ? gid / uint32_t(np) : 0u;
            if (np <= 0 || int64_t(phys) >= p.peer_slots) {
              if (chunk == 0) atomicOr(p.status, kStatusBadRemoteSlot);
            } else {
              ksrc = p.peer_k[bank] + int64_t(phys) * p.peer_stride;
              vsrc = p.peer_v[bank] + int64_t(phys) * p.peer_stride;
            }
          }
        }
        const int64_t off = h * 256 + chunk * 16;
        const uint32_t dst = tc::sw128_offset<kBN>(row, chunk);
        cp_async_16_zfill(sk + dst, ksrc + off, valid);
        cp_async_16_zfill(sv + dst, vsrc + off, valid);
      }
      // arrive on kv_full when this thread's copies of the tile have landed; keep issuing ahead
      cp_async_mbar_arrive_noinc(kv_full + s);
    }
    (void)ok;
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kMmaWarp) {
    // ================================================================ MMA issue (one thread)
    if (lane == 0) {
      constexpr uint32_t kIdescQK = tc::idesc_bf16_f32(128, kBN, 0, 0);
      constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t q_base = smem_addr(smem + kOffQ);
      const uint32_t kv_base = smem_addr(smem + kOffKV);
      auto issue_pv = [&](int q, int jj) {
        const uint32_t v_base = kv_base + (jj % kNS) * 2 * kKVBytes + kKVBytes;
        const uint32_t ph = tmem + kColP + q * 64, pl = ph + 32;  // 16 bf16 of K = 8 columns per MMA
        const uint32_t tO = tmem + 128 + q * 128;
#pragma unroll
        for (int kb = 0; kb < kBN / 16; ++kb) {
          const uint64_t vdesc = tc::smem_desc_sw128(v_base + kb * 2048, kBN * 128, 1024);
          tc::mma_bf16_ts(tO, ph + kb * 8, vdesc, kIdescPV, (jj > 0 || kb > 0) ? 1u : 0u);
          tc::mma_bf16_ts(tO, pl + kb * 8, vdesc, kIdescPV, 1u);
        }
        tc::commit(o_done + q);
      };
      bool ok = wait(q_full, 0);
      for (int j = 0; j < ntiles && ok; ++j) {
        const int s = j % kNS;
        if (!wait(kv_full + s, uint32_t(j / kNS) & 1u)) {
          ok = false;
          break;
        }
        fence_proxy_async_smem();
        tc::fence_after_sync();
        const uint32_t k_base = kv_base + s * 2 * kKVBytes;
        for (int q = 0; q < kQTiles; ++q) {
          if (j > 0) {  // softmax of (q, j-1) done: S_q is free and P_q(j-1) is ready
            if (!wait(p_full + q, uint32_t(j - 1) & 1u)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
          }
          const uint32_t qb = q_base + q * kQBytes;
#pragma unroll
          for (int kb = 0; kb < 8; ++kb) {
            const uint32_t off_q = (kb >> 2) * (kRows * 128) + (kb & 3) * 32;
            const uint32_t off_k = (kb >> 2) * (kBN * 128) + (kb & 3) * 32;
            tc::mma_bf16(tmem + q * kBN, tc::smem_desc_sw128(qb + off_q, 16, 1024),
                         tc::smem_desc_sw128(k_base + off_k, 16, 1024), kIdescQK, kb > 0);
          }
          tc::commit(s_full + q);
          if (j > 0) issue_pv(q, j - 1);
        }
        if (ok && j > 0) tc::commit(kv_empty + (j - 1) % kNS);  // frees that stage once PV(., j-1) completes
      }
      for (int q = 0; q < kQTiles && ok && ntiles > 0; ++q) {
        if (!wait(p_full + q, uint32_t(ntiles - 1) & 1u)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        issue_pv(q, ntiles - 1);
      }
    }
  } else {
    // ================================================================ softmax warpgroups
    const int q = warp / 4;                 // query tile
    const int r = tid - q * kRows;          // row = TMEM lane
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + q * kBN + lane_base;
    const uint32_t tO = tmem + 128 + q * 128 + lane_base;
    const int64_t tok_first = t_begin + q * kQTok;           // first token of this query tile
    const int64_t tok = tok_first + r / kGqa;
    const bool row_valid = tok < t_end;
    const float scale = p.scale_log2;
    const uint32_t tPh = tmem + kColP + q * 64 + lane_base, tPl = tPh + 32;
    float m_used = -INFINITY, d_sum = 0.f;  // m_used in the scaled (log2) domain
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      // warp-uniform decisions keep every warp-collective tcgen05.ld/st converged
      if (!__all_sync(0xffffffffu, wait(s_full + q, uint32_t(j) & 1u))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float x[kBN];
      tc::ld32(tS, x);
      tc::ld32(tS + 32, x + 32);
      tc::wait_ld();
      const int64_t base_pos = int64_t(j) * kBN;
      // a tile needs a mask only if it reaches past the end or across this query tile's diagonal
      const bool needs_mask =
          base_pos + kBN > kv_end || (p.causal && base_pos + kBN > prefix + tok_first + 1) || !row_valid;
      float tmax = -INFINITY;
      if (__any_sync(0xffffffffu, needs_mask)) {
        const int64_t lim = (row_valid && p.causal) ? min(kv_end, prefix + tok + 1) : kv_end;
        const int vis = int(max(int64_t(0), min(int64_t(kBN), lim - base_pos)));
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          x[c] = c < vis ? x[c] : -INFINITY;
          tmax = fmaxf(tmax, x[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBN; ++c) tmax = fmaxf(tmax, x[c]);
      }
      tmax *= scale;
      float alpha = 1.f;
      bool rescale = false;
      if (tmax > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - tmax);  // 0 on the first tile
        m_used = tmax;
        rescale = true;
      }
      // P_q and O_q are still in use by PV(q, j-1) until o_done
      if (j > 0 && !__all_sync(0xffffffffu, wait(o_done + q, uint32_t(j - 1) & 1u))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const float neg_m = -m_used;
      float rs = 0.f;
      uint32_t hi[kBN / 2], lo[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float p0 = fast_exp2(fmaf(x[c], scale, neg_m));
        const float p1 = fast_exp2(fmaf(x[c + 1], scale, neg_m));
        rs += p0 + p1;
        split_bf16x2(p0, p1, hi[c / 2], lo[c / 2]);
      }
      tc::st32u(tPh, hi);
      tc::st32u(tPl, lo);
      d_sum = d_sum * alpha + rs;
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float a = rescale ? alpha : 1.f;
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          float o[32];
          tc::ld32(tO + c0, o);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= a;
          tc::st32(tO + c0, o);
        }
        tc::wait_st();
      }
      tc::wait_st();  // P (and any rescaled O) in tensor memory before the MMA thread reads them
      tc::fence_before_sync();
      mbar_arrive(p_full + q);
    }
    // ---- epilogue: after the last PV of this query tile
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, wait(o_done + q, uint32_t(ntiles - 1) & 1u));
    tc::fence_after_sync();
    if (ok) {
      const float inv = d_sum > 0.f ? 1.f / d_sum : 0.f;
      __nv_bfloat16* dst = p.out + (q0 + (row_valid ? tok : 0)) * p.out_stride_tok +
                           int64_t(h * kGqa + r % kGqa) * p.out_stride_head;
#pragma unroll
      for (int c0 = 0; c0 < 128; c0 += 32) {
        float o[32];
        tc::ld32(tO + c0, o);
        tc::wait_ld();
        if (row_valid) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 packed;
            packed.x = pack_bf16x2(o[e] * inv, o[e + 1] * inv);
            packed.y = pack_bf16x2(o[e + 2] * inv, o[e + 3] * inv);
            packed.z = pack_bf16x2(o[e + 4] * inv, o[e + 5] * inv);
            packed.w = pack_bf16x2(o[e + 6] * inv, o[e + 7] * inv);
            *reinterpret_cast<uint4*>(dst + c0 + e) = packed;
          }
        }
      }
      if (row_valid && p.lse != nullptr)
        p.lse[(q0 + tok) * kNumQoHeads + h * kGqa + r % kGqa] = m_used + log2f(d_sum);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    if (*abort_flag) {
      // an aborted CTA may still have MMAs in flight: give them a bounded chance before TMEM goes
      for (int q = 0; q < kQTiles; ++q) {
        mbar_wait_bounded(o_done + q, 0);
        mbar_wait_bounded(o_done + q, 1);
      }
    }
    tc::dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int64_t append_plan(const int32_t* qo_indptr, const int32_t* kv_indptr, int batch, int causal, int32_t* work,
                    int64_t max_work) {
  struct Item {
    int64_t cost;
    int b, h, pair;
  };
  std::vector<Item> items;
  for (int b = 0; b < batch; ++b) {
    const int64_t q_len = int64_t(qo_indptr[b + 1]) - qo_indptr[b];
    const int64_t L = int64_t(kv_indptr[b + 1]) - kv_indptr[b];
    const int64_t prefix = L - q_len;
    for (int64_t t = 0; t < q_len; t += kPairTok) {
      const int64_t t_end = std::min(q_len, t + kPairTok);
      const int64_t kv_end = causal ? std::min(L, prefix + t_end) : L;
      const int64_t cost = (kv_end + kBN - 1) / kBN;
      for (int h = 0; h < kNumKvHeads; ++h) items.push_back({cost, b, h, int(t / kPairTok)});
    }
  }
  std::stable_sort(items.begin(), items.end(), [](const Item& a, const Item& c) { return a.cost > c.cost; });
  const int64_t n = int64_t(items.size());
  if (work != nullptr) {
    for (int64_t i = 0; i < n && i < max_work; ++i) {
      work[4 * i + 0] = items[i].b;
      work[4 * i + 1] = items[i].h;
      work[4 * i + 2] = items[i].pair;
      work[4 * i + 3] = int32_t(std::min<int64_t>(items[i].cost, 0x7fffffff));
    }
  }
  return n;
}

cudaError_t launch_tiered_append(const AppendParams& p, cudaStream_t stream) {
  if (p.num_work <= 0) return cudaSuccess;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tiered_append_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  tiered_append_kernel<<<p.num_work, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
