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
// Arithmetic follows the reference's append kernel
// (final/vendor/nvlink_prefill/launch_20261031_r5/code/paged_prefill.py:36-57): scores
// scaled into the log2 domain, online softmax in fp32, and P entering P @ V as a bf16
// high part plus the bf16 residual p - high (PROB_RESIDUAL, on by default there) -- here on work
// items with short rows (kResidualMaxEntries), where the parity bar needs it.
//
// Design (one CTA per work item = request x kv head x 64 query tokens, warp-specialised):
//   * two query tiles of 32 tokens x 4 GQA heads = 2 x 128 MMA rows share every K/V tile;
//     kv tiles are 128 entries: a tcgen05.mma of K = 16 costs the same ~76 cycles for any
//     N <= 128, so N = 128 score tiles halve the QK^T instructions per key against N = 64;
//   * loader warps (4, one per SM sub-partition; with 2 the gathers paced the kernel) gather K
//     and V tiles (128 entries x 256 B of this kv head, local HBM or a supplier's HBM through
//     peer loads) with 16-byte cp.async, 16 lanes per entry so every warp instruction moves
//     whole cache lines, into a 5-slot ring of 32 KB 128B-swizzled tiles filled in the order
//     K0 V0 K1 V1 ...; each loader arrives on the slot's barrier when its copies land
//     (cp.async.mbarrier.arrive), so loads run ahead of the tensor core;
//   * one MMA warp (one elected lane) issues, per kv tile j and query tile q:
//     O_q += P_q(j-1) V(j-1) (hi, and lo where the residual is on; A operand read from tensor
//     memory) and then S_q = Q_q K(j)^T into the same TMEM columns
//     (tcgen05.mma instructions of one thread execute in issue order, so the PV reads P before
//     the next QK overwrites it); one commit per query tile and kv tile tells the softmax both
//     that S_q(j) is ready and that O_q is quiescent;
//   * one softmax warpgroup per query tile (thread = TMEM lane = row): mask only on tiles that
//     cross the causal diagonal or the end, scale + exp2 as one FMA + one MUFU per score, lazy
//     rescaling of O in place (the reference max moves only when it grows by more than 2^8),
//     P written over its own S columns as bf16 hi/lo pairs (tcgen05.st); epilogue
//     O / rowsum -> bf16, LSE = m + log2 rowsum.
// All waits are bounded; a timed-out wait records DUAL_STATUS_WAIT_TIMEOUT and every role
// unwinds (no thread is left at a barrier the others skipped).
#include <algorithm>
#include <type_traits>
#include <vector>

#include "dual_b200.h"
#include "decode.cuh"
#include "prefill.cuh"
#include "tcgen05.cuh"

namespace dual {
namespace {

constexpr int kQTok = 32;                  // query tokens per query tile
constexpr int kRows = kQTok * kGqa;        // 128 MMA rows per query tile
constexpr int kQTiles = 2;                 // query tiles per CTA
constexpr int kPairTok = kQTok * kQTiles;  // 64 query tokens per work item
constexpr int kBN = 128;                   // kv entries per kv tile
constexpr int kSlots = 5;                  // ring slots, each one K or one V tile
constexpr int kLoadWarps = 4;
constexpr int kLoadThreads = kLoadWarps * 32;
constexpr int kWarpEntries = kBN / kLoadWarps;  // kv entries of a tile each loader warp gathers
constexpr int kLaneEntries = kWarpEntries / 32;  // entries whose row pointers one lane resolves
static_assert(kLaneEntries == 1 || kLaneEntries == 2, "loader warps gather 32 or 64 entries of a tile");
constexpr int kSoftmaxWarps = 4 * kQTiles;
constexpr int kMmaWarp = kSoftmaxWarps + kLoadWarps;  // the last warp
constexpr int kThreads = (kMmaWarp + 1) * 32;          // 416
constexpr float kRescaleThreshold = 8.0f;  // log2 units: p stays <= 256 between rescales
// P enters P @ V as a bf16 high part plus its bf16 residual only in work items whose shortest query
// row sees fewer than this many kv entries.  Rounding P to bf16 costs up to 2^-9 of each term; on
// short rows, where a few keys of opposite sign can cancel, that exceeds the 2e-3 / 1e-2 parity bar
// (the reference's validation shapes of 1..100 entries: 1.2-1.5x the bar), while rows of 512 entries
// and more stay below 0.3x of it, falling with length (fp32 oracle, N(0,1) inputs).  Longer rows
// therefore round P like FlashInfer's FA2: the residual is neither stored nor multiplied (a third of
// the tensor work on the 4-GPU append shapes).
constexpr int64_t kResidualMaxEntries = 1024;

constexpr int kQBytes = kRows * 256;       // 32 KB: [128 rows x 128 dims] bf16
constexpr int kSlotBytes = kBN * 256;      // 32 KB: [128 entries x 128 dims] bf16
// smem: Q0 Q1 | kSlots x (K or V tile) | barriers
constexpr int kOffQ = 0;
constexpr int kOffSlot = kQTiles * kQBytes;
constexpr int kOffBar = kOffSlot + kSlots * kSlotBytes;
constexpr int kNumBars = 2 * kSlots + 4 * kQTiles + 1;
constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

// TMEM columns: S0/P0 [0,128) S1/P1 [128,256) O0 [256,384) O1 [384,512).
// P of kv chunk c (entries 32c..32c+31) lives over S columns [32c, 32c+32): bf16 pairs, hi in the
// first 16 columns, lo in the last 16, so each chunk's P only overwrites scores already read.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;

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
  uint64_t* slot_full = bars;                    // [kSlots] count kLoadThreads
  uint64_t* slot_empty = bars + kSlots;          // [kSlots] count 1 (tcgen05.commit)
  uint64_t* s_full = bars + 2 * kSlots;          // [2]      count 1 (tcgen05.commit)
  uint64_t* p_part = s_full + kQTiles;           // [2 x 2]  count 128: P of entries 32..127, then 0..31
  uint64_t* o_done = p_part + 2 * kQTiles;       // [2]      count 1 (tcgen05.commit, last PV)
  uint64_t* q_full = o_done + kQTiles;           // [1]      count kLoadThreads
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kNumBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars) + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 w = p.work[blockIdx.x];
  const int b = w.x, h = w.y, pair = w.z;
  if (b < 0 || b >= p.batch || h < 0 || h >= kNumKvHeads || pair < 0) {  // a work list from another plan
    if (tid == 0) atomicOr(p.status, kStatusBadLength);
    return;
  }
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
  const bool use_lo = (p.causal ? prefix + t_begin + 1 : L) < kResidualMaxEntries;  // CTA-uniform

  // supplier bank pointers in shared memory: the loaders index them by bank at run time, and
  // indexing the kernel's parameter block instead would make every parameter a memory operand
  // that each asm statement with a memory clobber forces the compiler to reload
  __shared__ const char* s_peer[2][kMaxPeers];
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < kMaxPeers; ++i) {  // constant indices: plain parameter loads
      s_peer[0][i] = p.peer_k[i];
      s_peer[1][i] = p.peer_v[i];
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(slot_full + s, kLoadThreads);
      mbar_init(slot_empty + s, 1);
    }
    for (int q = 0; q < kQTiles; ++q) {
      mbar_init(s_full + q, 1);
      mbar_init(p_part + 2 * q, kRows);
      mbar_init(p_part + 2 * q + 1, kRows);
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

  // fast path first: under the tensor core's operand traffic every shared-memory access of a
  // waiting thread is slow, so the abort flag is read only when the phase is not complete yet
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity)) return true;
    *abort_flag = 1;
    atomicOr(p.status, kStatusWaitTimeout);
    return false;
  };

  if (warp >= kSoftmaxWarps && warp < kMmaWarp) {
    // ================================================================ loaders
    const int lt = tid - kSoftmaxWarps * 32;  // 0 .. kLoadThreads - 1
    // query tiles: 256 rows x 16 chunks of 16 B over the loader threads
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
    // kv tiles: loader warp lw owns entries [E lw, E lw + E) of each tile (E = kWarpEntries).  Lane l
    // resolves the page ids of entries E lw + 32 e + l into K and V row pointers one tile ahead of
    // use (the ids themselves are loaded two tiles ahead); the copy loop then only shuffles a
    // pointer: 16 lanes cover one entry's 256 B (two full 128 B lines), so each warp-wide cp.async
    // moves two entries, coalesced.  Resolving inside the copy loop (the remote branch with its
    // division and status update once per copy) made the loop four times slower.
    const int lw = lt >> 5;
    const int half = lane >> 4, chunk = lane & 15;
    const int32_t* const indices = p.indices + kv0;
    const char* const k_local = p.k_local;
    const char* const v_local = p.v_local;
    const int64_t local_stride = p.local_stride, peer_stride = p.peer_stride, peer_slots = p.peer_slots;
    const uint32_t capacity = static_cast<uint32_t>(p.local_capacity);
    const uint32_t np = static_cast<uint32_t>(max(p.num_peers, 0));
    unsigned* const status = p.status;
    const int64_t off = h * 256 + chunk * 16;
    auto page_of = [&](int jj, int sub) -> int32_t {  // page id of entry E lw + 32 sub + lane (0 past the end)
      const int64_t pos = int64_t(jj) * kBN + kWarpEntries * lw + 32 * sub + lane;
      return pos < kv_end ? __ldg(indices + pos) : 0;
    };
    // page id -> row pointers of both planes (page 0 of the local pool for a bad remote id, which is
    // recorded in the status word)
    auto resolve = [&](int32_t page_id, const char*& kp, const char*& vp) {
      const uint32_t page = static_cast<uint32_t>(page_id);
      if (page <= capacity) {
        kp = k_local + int64_t(page) * local_stride;
        vp = v_local + int64_t(page) * local_stride;
      } else {
        const uint32_t gid = page - capacity - 1u;
        const uint32_t bank = np > 0 ? gid % np : 0u;
        const uint32_t phys = np > 0 ? gid / np : 0u;
        if (np == 0 || int64_t(phys) >= peer_slots) {
          atomicOr(status, kStatusBadRemoteSlot);
          kp = k_local;
          vp = v_local;
        } else {
          kp = s_peer[0][bank] + int64_t(phys) * peer_stride;
          vp = s_peer[1][bank] + int64_t(phys) * peer_stride;
        }
      }
    };
    const char *kr[kLaneEntries], *vr[kLaneEntries];  // row pointers of this lane's entries, current tile
    int32_t next[kLaneEntries];
#pragma unroll
    for (int e = 0; e < kLaneEntries; ++e) {
      resolve(page_of(0, e), kr[e], vr[e]);
      next[e] = ntiles > 1 ? page_of(1, e) : 0;
    }
    auto shfl_ptr = [](const char* ptr, int src_lane) {
      const unsigned long long v = reinterpret_cast<unsigned long long>(ptr);
      const uint32_t lo = __shfl_sync(0xffffffffu, static_cast<uint32_t>(v), src_lane);
      const uint32_t hi = __shfl_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), src_lane);
      return reinterpret_cast<const char*>((static_cast<unsigned long long>(hi) << 32) | lo);
    };
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      int32_t after[kLaneEntries];  // lands while this tile issues
#pragma unroll
      for (int e = 0; e < kLaneEntries; ++e) after[e] = j + 2 < ntiles ? page_of(j + 2, e) : 0;
      const int64_t tile0 = int64_t(j) * kBN;
#pragma unroll 1
      for (int plane = 0; plane < 2; ++plane) {  // K then V of tile j
        const int u = 2 * j + plane, s = u % kSlots, f = u / kSlots;
        if (f > 0 && !wait(slot_empty + s, uint32_t(f - 1) & 1u)) {
          ok = false;
          break;
        }
        unsigned char* dst_tile = smem + kOffSlot + s * kSlotBytes;
#pragma unroll 8
        for (int i = 0; i < kWarpEntries / 2; ++i) {
          const int rr = 2 * i + half;  // entry within this warp's share
          const int row = kWarpEntries * lw + rr;
          const char* const* rows = plane == 0 ? kr : vr;
          const char* src = shfl_ptr(kLaneEntries == 1 || i < 16 ? rows[0] : rows[kLaneEntries - 1], rr & 31);
          const bool valid = tile0 + row < kv_end;
          cp_async_16_zfill(dst_tile + tc::sw128_offset<kBN>(row, chunk), src + off, valid);
        }
        // arrive on the slot's barrier when this thread's copies have landed; keep issuing ahead
        // (a test injection withholds the first K tile's arrival: the consumers' waits expire)
        if (!(u == 0 && (p.inject & DUAL_INJECT_APPEND_WITHHOLD_K0))) cp_async_mbar_arrive_noinc(slot_full + s);
      }
#pragma unroll
      for (int e = 0; e < kLaneEntries; ++e) {
        if (j + 1 < ntiles) resolve(next[e], kr[e], vr[e]);
        next[e] = after[e];
      }
    }
    (void)ok;
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kMmaWarp) {
    // ================================================================ MMA issue (one warp, one lane)
    // Query tiles alternate (PV_0 QK_0, PV_1 QK_1), so the tensor core works on one tile while the
    // other is in softmax; within a tile PV_q(j-1) is issued before QK_q(j), which overwrites P_q.
    // The whole warp runs the loop in warp-uniform control flow (every wait is a warp vote), so the
    // descriptors and TMEM addresses are uniform values, and one elected lane issues each tcgen05
    // instruction.  Run by lane 0 alone inside a divergent branch, the same loop cost the issuing
    // thread ~100 cycles per MMA (traced with clock64 on config-4 shapes: 4 MMAs to an idle tensor
    // core took 400 cycles), and that issue rate, not the tensor core, set the kernel's pace.
    const bool leader = tc::elect_one();
    auto wait_warp = [&](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, wait(bar, parity)); };
    {
      constexpr uint32_t kIdescQK = tc::idesc_bf16_f32(128, kBN, 0, 0);
      constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t q_base = smem_addr(smem + kOffQ);
      const uint32_t slot_base = smem_addr(smem + kOffSlot);
      auto slot_addr = [&](int u) { return slot_base + uint32_t(u % kSlots) * kSlotBytes; };
      auto slot_wait = [&](int u) { return wait_warp(slot_full + u % kSlots, uint32_t(u / kSlots) & 1u); };
      // O_q (+)= P_q V(jj), k-steps of 16 entries, each a hi and a lo MMA with A from TMEM; part 0 is
      // entries 32..127 (k-steps 2..7, the first P the softmax writes), part 1 entries 0..31: the
      // smaller the last part, the fewer MMAs stand between the end of a softmax and the next QK
      // (96/32 against 64/64: 7.70-7.76 vs 7.81-7.84 ms on config 4, same box)
      auto issue_pv_part = [&](int q, int jj, int part) {
        const uint32_t v_base = slot_addr(2 * jj + 1);
        const uint32_t tP = tmem + q * kBN;
        const uint32_t tO = tmem + kColO + q * 128;
#pragma unroll
        for (int k = 0; k < (part == 0 ? 6 : 2); ++k) {
          const int kb = part == 0 ? 2 + k : k;
          const uint64_t vdesc = tc::smem_desc_sw128(v_base + kb * 2048, kBN * 128, 1024);
          const uint32_t ph = tP + 32 * (kb >> 1) + 8 * (kb & 1);
          if (leader) {
            tc::mma_bf16_ts(tO, ph, vdesc, kIdescPV, (jj > 0 || part > 0 || k > 0) ? 1u : 0u);
            if (use_lo) tc::mma_bf16_ts(tO, ph + 16, vdesc, kIdescPV, 1u);
          }
        }
      };
      // both parts of PV_q(jj), each once the softmax has written that part of P
      auto issue_pv = [&](int q, int jj) -> bool {
        for (int part = 0; part < 2; ++part) {
          if (!wait_warp(p_part + 2 * q + part, uint32_t(jj) & 1u)) return false;
          tc::fence_after_sync();
          issue_pv_part(q, jj, part);
        }
        return true;
      };
      bool ok = wait_warp(q_full, 0);
      for (int j = 0; j < ntiles && ok; ++j) {
        const uint32_t k_base = slot_addr(2 * j);
        // K(j) landed, and with it V(j-1): each loader thread issues V(j-1) before K(j) and arrives
        // on K(j)'s barrier only once all of its earlier copies have landed (one poll, not two)
        if (!slot_wait(2 * j)) {
          ok = false;
          break;
        }
        fence_proxy_async_smem();  // cp.async writes -> tensor core reads
        tc::fence_after_sync();
        for (int q = 0; q < kQTiles; ++q) {
          if (j > 0 && !issue_pv(q, j - 1)) {  // P_q(j-1) is in TMEM, in two parts
            ok = false;
            break;
          }
          const uint32_t qb = q_base + q * kQBytes;
#pragma unroll
          for (int kb = 0; kb < 8; ++kb) {
            const uint32_t off_q = (kb >> 2) * (kRows * 128) + (kb & 3) * 32;
            const uint32_t off_k = (kb >> 2) * (kBN * 128) + (kb & 3) * 32;
            if (leader)
              tc::mma_bf16(tmem + q * kBN, tc::smem_desc_sw128(qb + off_q, 16, 1024),
                           tc::smem_desc_sw128(k_base + off_k, 16, 1024), kIdescQK, kb > 0);
          }
          if (leader) tc::commit(s_full + q);  // S_q(j) written, PV_q(j-1) done
        }
        if (!ok) break;
        if (leader) {
          tc::commit(slot_empty + (2 * j) % kSlots);                 // K(j) consumed by both QKs
          if (j > 0) tc::commit(slot_empty + (2 * j - 1) % kSlots);  // V(j-1) consumed by both PVs
        }
      }
      if (ok && ntiles > 0) {
        ok = slot_wait(2 * ntiles - 1);
        if (ok) fence_proxy_async_smem();
      }
      for (int q = 0; q < kQTiles && ok && ntiles > 0; ++q) {
        if (!issue_pv(q, ntiles - 1)) break;
        if (leader) tc::commit(o_done + q);
      }
    }
  } else {
    // ================================================================ softmax warpgroups
    const int q = warp / 4;                 // query tile
    const int r = tid - q * kRows;          // row = TMEM lane
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + q * kBN + lane_base;
    const uint32_t tO = tmem + kColO + q * 128 + lane_base;
    const int64_t tok_first = t_begin + q * kQTok;           // first token of this query tile
    const int64_t tok = tok_first + r / kGqa;
    const bool row_valid = tok < t_end;
    const float scale = p.scale_log2;
    const bool causal = p.causal != 0;
    float m_used = -INFINITY, d_sum = 0.f;  // m_used in the scaled (log2) domain
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      // warp-uniform decisions keep every warp-collective tcgen05.ld/st converged
      if (!__all_sync(0xffffffffu, wait(s_full + q, uint32_t(j) & 1u))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const int64_t base_pos = int64_t(j) * kBN;
      // a tile needs a mask only if it reaches past the end or across this query tile's diagonal
      const bool needs_mask = __any_sync(
          0xffffffffu,
          base_pos + kBN > kv_end || (causal && base_pos + kBN > prefix + tok_first + 1) || !row_valid);
      const int64_t lim = (row_valid && causal) ? min(kv_end, prefix + tok + 1) : kv_end;
      const int vis = int(max(int64_t(0), min(int64_t(kBN), lim - base_pos)));  // visible entries
      // scores in two halves of 64 columns (64 live registers): max over both, the second half
      // stays live for the exponentials and the first half is read again afterwards
      float x[64];
      auto load_half = [&](int c0) {
        tc::ld32(tS + c0, x);
        tc::ld32(tS + c0 + 32, x + 32);
        tc::wait_ld();
        if (needs_mask) {
#pragma unroll
          for (int c = 0; c < 64; ++c) x[c] = c0 + c < vis ? x[c] : -INFINITY;
        }
      };
      auto half_max = [&]() {  // four independent chains of three-input maxima
        float m4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
        for (int c = 4; c < 60; c += 8) {
#pragma unroll
          for (int e = 0; e < 4; ++e) m4[e] = fmax3(m4[e], x[c + e], x[c + 4 + e]);
        }
        return fmax3(fmax3(m4[0], m4[1], x[60]), fmax3(m4[2], m4[3], x[61]), fmaxf(x[62], x[63]));
      };
      load_half(0);
      float tmax = half_max();
      load_half(64);
      tmax = fmaxf(tmax, half_max()) * scale;
      float alpha = 1.f;
      bool rescale = false;
      if (tmax > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - tmax);  // 0 on the first tile
        m_used = tmax;
        rescale = true;
      }
      // O_q is quiescent here: PV_q(j-1) completed before s_full(j), PV_q(j) waits for this P
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float a = rescale ? alpha : 1.f;
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          float o[32];
          tc::ld32(tO + c0, o);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= a;
          tc::st32(tO + c0, o);
        }
      }
      const uint64_t scale2 = f2_pack(scale, scale), neg_m2 = f2_pack(-m_used, -m_used);
      // packed partial row sums, four independent chains: warps issue in order, and with two chains
      // the dependent adds stalled the exponentials behind them (one warp alone: 545 -> 378 cycles per
      // 32 scores in a clock64 probe of this loop on a B200)
      uint64_t rs2[4] = {0, 0, 0, 0};
      // P of 32 entries written over their own S columns: [0,16) hi pairs, [16,32) lo pairs.
      // hi = rn_bf16(p), lo = rn_bf16(p - hi), with the scale, the sums and the residual on packed
      // f32x2 arithmetic.
      auto emit_p = [&](const float* xc, int col, auto lo_tag) {
        constexpr bool kLo = decltype(lo_tag)::value;
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {  // 16 entries: 8 hi words, 8 lo words
          uint32_t hi[8], lo[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float t0, t1;
            f2_unpack(f2_fma(f2_pack(xc[16 * sub + 2 * i], xc[16 * sub + 2 * i + 1]), scale2, neg_m2), t0, t1);
            const float p0 = fast_exp2(t0), p1 = fast_exp2(t1);
            const uint64_t pp = f2_pack(p0, p1);
            rs2[i & 3] = f2_add(rs2[i & 3], pp);
            hi[i] = pack_bf16x2(p0, p1);
            if (kLo) {  // the residual only where it is multiplied (1.7 % of a config-4 layer)
              const uint64_t hh = f2_pack(__uint_as_float(hi[i] << 16), __uint_as_float(hi[i] & 0xffff0000u));
              float l0, l1;
              f2_unpack(f2_sub(pp, hh), l0, l1);
              lo[i] = pack_bf16x2(l0, l1);
            }
          }
          tc::st8u(tS + col + 8 * sub, hi);
          if (kLo) tc::st8u(tS + col + 16 + 8 * sub, lo);
        }
      };
      auto emit = [&](const float* xc, int col) {
        if (use_lo)
          emit_p(xc, col, std::true_type{});
        else
          emit_p(xc, col, std::false_type{});
      };
      auto mask32 = [&](float* xc, int col) {
        if (needs_mask) {
#pragma unroll
          for (int c = 0; c < 32; ++c) xc[c] = col + c < vis ? xc[c] : -INFINITY;
        }
      };
      // x holds entries 64..127; entries 0..63 are read again into each half of x once it is
      // consumed, overlapping the exponentials.  P of entries 32..127 goes to the MMA warp as soon
      // as it is in tensor memory (with any rescaled O before it), then P of entries 0..31.
      emit(x, 64);
      tc::ld32(tS, x);
      emit(x + 32, 96);
      tc::ld32(tS + 32, x + 32);
      tc::wait_ld();
      mask32(x + 32, 32);
      emit(x + 32, 32);
      tc::wait_st();
      tc::fence_before_sync();
      mbar_arrive(p_part + 2 * q);
      mask32(x, 0);
      emit(x, 0);
      float r0, r1, r2, r3;
      f2_unpack(f2_add(rs2[0], rs2[1]), r0, r1);
      f2_unpack(f2_add(rs2[2], rs2[3]), r2, r3);
      d_sum = d_sum * alpha + ((r0 + r1) + (r2 + r3));
      tc::wait_st();
      tc::fence_before_sync();
      mbar_arrive(p_part + 2 * q + 1);
    }
    // ---- epilogue: after the last PV of this query tile
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, wait(o_done + q, 0));
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
        mbar_wait_bounded(s_full + q, 0);
        mbar_wait_bounded(s_full + q, 1);
      }
    }
    tc::dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// Work items (request, kv head, 64-token query pair), in launch order: (request, kv head) groups
// longest first, and within a group its pairs longest first.  CTAs launched together then belong to
// the same group and stream the same K/V rows, which stay in L2 for all but the first of them
// (ordering the items by cost alone interleaves groups, and on the 4-GPU append shapes every K/V
// row was read from DRAM ~4.3 times); the pairs of a group differ in cost by at most
// q / 128 tiles, so the order stays close to longest-processing-time-first.
//
// With per-request remote counts, the items of requests whose list is mostly remote (share above
// kSpreadRemoteShare) are spread evenly over the first kSpreadSpan of the launch order, longest
// first, between the others.  A peer's rows are not cached in this GPU's L2, so every item of such a
// request reads its rows over NVLink again; launched together (as the grouped order would), the
// items of the ~95 %-remote requests of the 4-GPU append shapes saturate NVLink ingress while the
// rest of the GPU waits (12.6 ms per layer with the banks on a peer), spread out they share it with
// compute-bound items (9.26 ms, against 9.19 ms with the rows staged into local memory first).
namespace {
constexpr double kSpreadRemoteShare = 0.5;
constexpr double kSpreadSpan = 0.9;
}  // namespace

int64_t append_plan(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* remote, int batch, int causal,
                    int32_t* work, int64_t max_work) {
  struct Group {
    int64_t cost;
    int b, h;
  };
  struct Item {
    int32_t b, h, t, tiles;
  };
  std::vector<Group> groups;
  for (int b = 0; b < batch; ++b) {
    const int64_t q_len = int64_t(qo_indptr[b + 1]) - qo_indptr[b];
    const int64_t L = int64_t(kv_indptr[b + 1]) - kv_indptr[b];
    if (q_len <= 0) continue;
    const int64_t cost = (L + kBN - 1) / kBN;  // the group's last pair sees the whole list, causal or not
    for (int h = 0; h < kNumKvHeads; ++h) groups.push_back({cost, b, h});
  }
  std::stable_sort(groups.begin(), groups.end(), [](const Group& a, const Group& c) { return a.cost > c.cost; });
  auto heavy = [&](int b) {
    const int64_t L = int64_t(kv_indptr[b + 1]) - kv_indptr[b];
    return remote != nullptr && L > 0 && double(remote[b]) > kSpreadRemoteShare * double(L);
  };
  std::vector<Item> light, spread;
  for (const Group& g : groups) {
    const int64_t q_len = int64_t(qo_indptr[g.b + 1]) - qo_indptr[g.b];
    const int64_t L = int64_t(kv_indptr[g.b + 1]) - kv_indptr[g.b];
    const int64_t prefix = L - q_len;
    const int64_t pairs = (q_len + kPairTok - 1) / kPairTok;
    for (int64_t t = pairs - 1; t >= 0; --t) {  // longest pair first
      const int64_t t_end = std::min(q_len, (t + 1) * kPairTok);
      const int64_t kv_end = causal ? std::min(L, prefix + t_end) : L;
      const Item it{g.b, g.h, int32_t(t), int32_t(std::min<int64_t>((kv_end + kBN - 1) / kBN, 0x7fffffff))};
      (heavy(g.b) ? spread : light).push_back(it);
    }
  }
  std::stable_sort(spread.begin(), spread.end(), [](const Item& a, const Item& c) { return a.tiles > c.tiles; });
  const int64_t n = int64_t(light.size() + spread.size());
  if (work == nullptr) return n;
  // merge: the k-th spread item goes at position floor(k * span * n / |spread|) or the first free one after
  size_t li = 0, si = 0;
  for (int64_t i = 0; i < n && i < max_work; ++i) {
    bool take_spread = si < spread.size() &&
                       (li >= light.size() || double(i) >= double(si) * kSpreadSpan * double(n) / double(spread.size()));
    const Item& it = take_spread ? spread[si++] : light[li++];
    work[4 * i + 0] = it.b;
    work[4 * i + 1] = it.h;
    work[4 * i + 2] = it.t;
    work[4 * i + 3] = it.tiles;
  }
  return n;
}

cudaError_t launch_tiered_append(const AppendParams& p, cudaStream_t stream) {
  if (p.num_work <= 0) return cudaSuccess;
  static std::atomic<uint64_t> configured{0};
  if (cudaError_t e = set_max_dynamic_smem_once(tiered_append_kernel, kSmemBytes, configured)) return e;
  tiered_append_kernel<<<p.num_work, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dual
