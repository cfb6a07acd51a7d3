/*
 * dual_b200 C ABI -- the drop-in boundary of the tiered-KV hot path.
 *
 * Plain pointers and sizes only; every call is asynchronous on the given CUDA
 * stream (a cudaStream_t passed as void*, NULL = legacy default stream) and is
 * safe to capture in a CUDA graph unless stated otherwise.  Every function
 * returns 0 on success or a nonzero DUAL_E* code, in which case
 * dual_last_error() returns a thread-local message.  Device-side problems
 * (bad page ids, timed-out waits) are recorded as bits in a caller-provided
 * 32-bit device status word (see DUAL_STATUS_*), never as traps.
 *
 * Model constants fixed by the reference (Qwen3-8B layer, page_size 1):
 * 32 query heads, 8 kv heads, head_dim 128, bf16 KV, NHD layout.
 */
#ifndef DUAL_B200_H
#define DUAL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ error codes */
#define DUAL_OK 0
#define DUAL_EINVAL 1     /* bad argument (shape, null pointer, alignment) */
#define DUAL_ECUDA 2      /* a CUDA runtime call failed */
#define DUAL_ENOSPACE 3   /* workspace too small */
#define DUAL_EUNSUPPORTED 4

/* device status bits (written by kernels into the caller's status word) */
#define DUAL_STATUS_BAD_LOCAL_SLOT 0x1u
#define DUAL_STATUS_BAD_REMOTE_SLOT 0x2u
#define DUAL_STATUS_WAIT_TIMEOUT 0x4u
#define DUAL_STATUS_BAD_COPY_SLOT 0x8u
#define DUAL_STATUS_BAD_LENGTH 0x10u
#define DUAL_STATUS_BAD_TIER 0x20u

/* Thread-local message of the last failing call ("" if none). */
const char* dual_last_error(void);
/* ABI version of this library (major * 100 + minor): 200 = the merge inside the decode kernel (a
 * workspace with arrival counters, dual_decode_workspace_reset). */
int dual_abi_version(void);

/* ------------------------------------------------------- tiered decode ---
 * Replaces the patched FlashInfer FA2 batch-prefill module used for decode:
 *   peer/flashinfer_peer.py:27-78   paged_kv_t::tiered_address (page-id resolver)
 *   peer/flashinfer_peer.py:105-142 module(): custom JIT with extra tensors
 *     peer_k0..peer_v2, unified_indices and scalars local_capacity, sm_scale
 *   peer/backend.py:132-138         wrapper.run(q, paged_kv, *peers, indices, C, scale)
 * Page id p in unified_indices: p <= local_capacity -> local slot p;
 * else g = p - local_capacity - 1 -> peer bank g % num_peers, slot g / num_peers.
 *
 * q           [batch, 32, 128] bf16, strides in elements (q_stride_head even)
 * k_local/v_local  local pool planes of one layer, slot p at base + p*local_stride_bytes,
 *             8 heads x 128 bf16 contiguous per slot (NHD, page_size 1)
 * peer_k/peer_v    host arrays of num_peers (0..8) device pointers (may be peer
 *             GPUs' memory mapped by IPC or peer access), same per-slot layout
 * kv_indptr   [batch+1] int32 device prefix sums of kv lengths
 * unified_indices  kv_indptr[batch] int32 page ids in read order; num_indices is the
 *             buffer's capacity (entries beyond it are never read: the status word
 *             records DUAL_STATUS_BAD_LENGTH and the tail is skipped)
 * out         [batch, 32, 128] bf16; lse [batch, 32] fp32 (base 2, FlashInfer's
 *             convention) or NULL
 * workspace   device scratch of >= dual_decode_workspace_size(batch, num_ctas)
 *             bytes, 256-byte aligned: [status word, 256 B][one arrival counter per
 *             (request, kv head)][partial softmax states].  Zero its head once with
 *             dual_decode_workspace_reset before the first call (or allocate it
 *             zeroed); launches leave the counters at zero again, so one reset per
 *             workspace is enough -- except after a launch whose status word shows
 *             DUAL_STATUS_WAIT_TIMEOUT or DUAL_STATUS_BAD_LENGTH, which may leave
 *             counters behind.  The status word is cleared by dual_status_clear or
 *             the reset, never by this call.
 * num_ctas    CTAs (0 = one per SM); fixed per graph capture
 * A request split over several CTAs is merged by the last of them to finish, inside the same
 * kernel (one launch per call).
 */
size_t dual_decode_workspace_size(int batch, int num_ctas);
/* Zeroes the status word and the arrival counters of a decode workspace for up to `batch` requests
 * (asynchronous on `stream`, capturable). */
int dual_decode_workspace_reset(void* workspace, size_t workspace_bytes, int batch, int device, void* stream);
int dual_decode_default_ctas(int device);
int dual_tiered_decode(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                       const void* k_local, const void* v_local, int64_t local_stride_bytes,
                       int64_t local_capacity,
                       const void* const* peer_k, const void* const* peer_v, int num_peers,
                       int64_t peer_stride_bytes, int64_t peer_slots,
                       const int32_t* kv_indptr, const int32_t* unified_indices, int64_t num_indices,
                       int batch, double sm_scale,
                       void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                       void* workspace, size_t workspace_bytes, int num_ctas,
                       int device, void* stream);

/* Allocation-free variant of dual_tiered_decode.  It has no counterpart in the reference:
 * it exists for callers that cannot allocate device memory or pass a workspace (a serving
 * process whose memory manager already owns almost all of HBM and forbids out-of-band
 * cudaMalloc, or a foreign-language binding that only holds the attention tensors).
 * The split-KV partial states live in a fixed 8 MiB file-scope device array that every
 * GPU loading this library holds until exit; (num_ctas + batch) * 16896 + 256 bytes plus
 * batch * 32 bytes of arrival counters (rounded up to 256) must fit in it (e.g. batch <= 347
 * with the default 148 CTAs), otherwise DUAL_ENOSPACE.  Each call zeroes the counters first.
 * All calls on a device share that array and it keeps the last call's contents: calls
 * that overlap on the GPU race on it.  The first call on a device looks up the array's
 * address (with that device current); make it before any stream capture.
 * status: NULL (this call clears the array's own status word and records into it; read it
 * back with dual_decode_noalloc_status before the next call on the device) or a caller-owned
 * device status word that kernels OR bits into.  Other arguments as for dual_tiered_decode,
 * device < 0 included (the calling thread's current device). */
int dual_tiered_decode_noalloc(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                               const void* k_local, const void* v_local, int64_t local_stride_bytes,
                               int64_t local_capacity,
                               const void* const* peer_k, const void* const* peer_v, int num_peers,
                               int64_t peer_stride_bytes, int64_t peer_slots,
                               const int32_t* kv_indptr, const int32_t* unified_indices,
                               int64_t num_indices, int batch, double sm_scale,
                               void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                               uint32_t* status, int num_ctas, int device, void* stream);
/* Part of the allocation-free decode above (no reference counterpart): copies the status word of
 * the device's scratch array -- the bits of the last dual_tiered_decode_noalloc call on `device`
 * that was given status == NULL -- to *value_out once the work queued on `stream` has finished.
 * Synchronous (not capturable); allocates nothing. */
int dual_decode_noalloc_status(uint32_t* value_out, int device, void* stream);

/* ------------------------------------------------------ tiered append ---
 * Replaces the tiered FA2 batch-prefill module on the append path (run hook
 * peer/prefill_backend.py:25-42, module peer/flashinfer_peer.py:105-142).  The banks passed as
 * peer_k / peer_v are read wherever they live: the suppliers' memory (peer loads) or local stage
 * buffers filled by dual_stage_bank_range / dual_stage_remote_rows.
 * Semantics of FlashInfer's BatchPrefillWithPagedKVCacheWrapper (page_size 1): request b has
 * qo_indptr[b+1]-qo_indptr[b] query tokens and kv_indptr[b+1]-kv_indptr[b] list entries; with
 * causal != 0 query token i sees entry j iff j < L_b - q_b (history, any order) or
 * j - (L_b - q_b) <= i (the query suffix, in order -- the packer's Full list).
 * dual_append_plan (host): from HOST copies of qo_indptr / kv_indptr, writes the work list
 * (4 int32 per item: request, kv head, 64-token query pair, 128-entry kv tiles), grouped by
 * (request, kv head) so a group's items run together and share K/V rows in L2, groups longest
 * first and pairs longest first within a group; returns the item count in *num_work (call with
 * work=NULL to size it).  remote_counts_host (NULL = unknown): per request, how many of its list
 * entries are on suppliers; the items of requests that are more than half remote are then spread
 * evenly over the first 90 % of the launch, longest first, so that their NVLink reads (a peer's rows
 * are not cached in the local L2, so every query pair reads them again) overlap compute-bound items
 * instead of saturating NVLink together.  The work list is then copied to
 * the device and passed to dual_tiered_append with the DEVICE indptrs.
 * q/out [sum q, 32, 128] bf16; lse [sum q, 32] fp32 base 2 or NULL; status: device word. */
int dual_append_plan(const int32_t* qo_indptr_host, const int32_t* kv_indptr_host, const int32_t* remote_counts_host,
                     int batch, int causal, int32_t* work_host, int64_t max_work, int64_t* num_work);
int dual_tiered_append(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                       const void* k_local, const void* v_local, int64_t local_stride_bytes,
                       int64_t local_capacity,
                       const void* const* peer_k, const void* const* peer_v, int num_peers,
                       int64_t peer_stride_bytes, int64_t peer_slots,
                       const int32_t* qo_indptr, const int32_t* kv_indptr,
                       const int32_t* unified_indices, int64_t num_indices, int batch, int causal,
                       double sm_scale, const int32_t* work, int64_t num_work,
                       void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
                       uint32_t* status, int device, void* stream);

/* ------------------------------------------------------ read-order packer ---
 * Replaces Triton _count_remote/_pack_indices + Engine.prepare (peer/backend.py:22-79)
 * and packing.prepare (peer/packing.py:6-36); exact order = peer/layout.py:5-22.
 * tier/slot   [table_rows, table_stride] int32 tables (tier 0 local / 1 remote / -1 unused);
 *             rows/positions outside them are skipped and flagged in status
 * prefix_lens NULL for decode (prefix = seq_lens) or [batch] for prefill/append
 * new_loc     NULL or [batch] int64: fused decode-step write of the newest token
 *             (slot[req, seq-1] = new_loc, tier = 0) before packing
 * full_out    sum(seq_lens) int32; history_out NULL or sum(prefix_lens) int32
 * status      NULL or a device status word
 */
int dual_pack_read_order(int32_t* tier, int32_t* slot, int64_t table_rows, int64_t table_stride,
                         const int32_t* req_pool_indices, const int32_t* seq_lens,
                         const int32_t* prefix_lens, const int64_t* new_loc, int batch,
                         int64_t local_capacity, int remote_rows, int tile_rows,
                         int32_t* full_out, int32_t* history_out, uint32_t* status,
                         int device, void* stream);

/* Replaces Triton _write_prefill_layout (peer/page_ops.py:6-18): for every request b and
 * j < length[b]: slot[req[b], prefix[b]+j] = locations[start[b]+j], tier[...] = 0.
 * locations are int64 (SGLang out_cache_loc) when loc_is_int64, else int32.  Writes outside the
 * [table_rows, table_stride] tables are skipped (status, when given, records DUAL_STATUS_BAD_LENGTH). */
int dual_write_prefill_layout(int32_t* tier, int32_t* slot, int64_t table_rows, int64_t table_stride,
                              const int32_t* req_pool_indices, const int32_t* start,
                              const int32_t* length, const int32_t* prefix,
                              const void* locations, int loc_is_int64, int batch, int max_length,
                              uint32_t* status, int device, void* stream);

/* Replaces SGLang's MHATokenToKVPool.set_kv_buffer as the reference calls it before every tiered
 * attention launch (V/nvlink_prefill_timing/backend.py:34,42): new positions are always local
 * (tier 0), so for i < n the K and V rows of token i (8 kv heads x 128 bf16, heads x dims
 * contiguous, token strides k_stride_token / v_stride_token in elements) are copied to slot
 * locations[i] of k_local / v_local (slot stride local_stride_bytes).  locations are int64 (SGLang
 * out_cache_loc) when loc_is_int64, else int32.  A slot outside [0, local_capacity] (0 is SGLang's
 * dummy slot) is skipped and records DUAL_STATUS_BAD_LOCAL_SLOT.  Bit-exact. */
int dual_set_kv_buffer(void* k_local, void* v_local, int64_t local_stride_bytes, int64_t local_capacity,
                       const void* k, int64_t k_stride_token, const void* v, int64_t v_stride_token,
                       const void* locations, int loc_is_int64, int64_t n, uint32_t* status, int device,
                       void* stream);

/* ------------------------------------------------------------- migration ---
 * Replaces Triton fused_copy._copy / copy_pages / restore (peer/fused_copy.py:6-33):
 * for each i < n and each plane: reverse==0 copies local slot source[i] to remote id
 * target[i] (bank target[i] % num_banks, slot target[i] / num_banks); reverse==1 copies
 * remote id source[i] to local slot target[i].  Bit-exact byte copy.
 * local_planes [num_planes] and remote_planes [num_banks*num_planes] are DEVICE int64
 * arrays of plane base pointers (RemoteBank.pointers layout, peer/remote_bank.py:23).
 * max_ctas bounds the SMs the copy occupies (0 = as many as rows need). */
int dual_migrate_copy(const int64_t* local_planes, const int64_t* remote_planes, int num_planes,
                      int num_banks, const int64_t* source, const int64_t* target, int64_t n,
                      int reverse, int64_t row_bytes, int64_t local_slots, int64_t remote_slots,
                      uint32_t* status, int max_ctas, int device, void* stream);

/* ------------------------------------------------------------ staging ---
 * Replaces LayerStager.launch (peer/staging.py:27-38), which copies every supplier bank's whole
 * layer into a local one-layer buffer before the prefill of that layer reads it
 * (peer/prefill_backend.py:33), selectively: for every entry p of unified_indices[0, num_indices)
 * with p > local_capacity (global remote id g = p - local_capacity - 1), copies row g / num_banks
 * of both planes of bank g % num_banks (peer_k[b], peer_v[b]: one layer's planes, bank_slots rows
 * at peer_stride_bytes) to the same row of stage_k[b] / stage_v[b] (local buffers, bank_slots rows
 * at stage_stride_bytes).  Local entries are skipped; rows no entry names are left untouched.  The
 * stage buffers then replace the banks in dual_tiered_append (or dual_tiered_decode) with the same
 * index list.  row_bytes (2048 for 8 kv heads x 128 x bf16) and the strides are multiples of 16.
 * A remote id beyond the banks is skipped and records DUAL_STATUS_BAD_REMOTE_SLOT.  max_ctas bounds
 * the grid (0 = one single-warp CTA per 32 entries). */
int dual_stage_remote_rows(const void* const* peer_k, const void* const* peer_v, void* const* stage_k,
                           void* const* stage_v, int num_banks, int64_t peer_stride_bytes,
                           int64_t stage_stride_bytes, int64_t bank_slots, int64_t row_bytes,
                           const int32_t* unified_indices, int64_t num_indices, int64_t local_capacity,
                           uint32_t* status, int max_ctas, int device, void* stream);

/* Row-range staging on the copy engines, the reference's form (LayerStager.launch copies each
 * donor's whole layer with one copy per donor on its own stream, peer/staging.py:27-38): for each
 * bank b with row_begin[b] < row_end[b], copies rows [row_begin[b], row_end[b]) of both planes from
 * peer_k/peer_v[b] to the same rows of stage_k/stage_v[b] -- one cudaMemcpyAsync per plane when
 * both strides equal row_bytes, else one cudaMemcpy2DAsync -- on streams[b] (host array of
 * num_banks stream handles; NULL entries mean the legacy default stream).  No SM work, so it
 * overlaps a running attention kernel.  Ranges must lie within [0, bank_slots]. */
int dual_stage_bank_range(const void* const* peer_k, const void* const* peer_v, void* const* stage_k,
                          void* const* stage_v, int num_banks, int64_t peer_stride_bytes,
                          int64_t stage_stride_bytes, int64_t bank_slots, int64_t row_bytes,
                          const int64_t* row_begin, const int64_t* row_end, void* const* streams, int device);

/* ------------------------------------------------------ fault injection ---
 * Test hook with no counterpart in the reference (whose failure handling is fail-fast asserts):
 * makes a device-side wait run out without faulting the GPU, so tests can check that the
 * bounded waits turn into DUAL_STATUS_WAIT_TIMEOUT and leave the context usable.  The mask is
 * process-wide host state read at launch; 0 (the default) disables every injection.
 *   DUAL_INJECT_APPEND_WITHHOLD_K0: tiered_append loaders never arrive on the barrier of their
 *   first K tile, so the MMA thread's wait for it expires (~1 s), every role unwinds, and each CTA
 *   records the timeout in the status word. */
#define DUAL_INJECT_APPEND_WITHHOLD_K0 0x1u
int dual_debug_inject(uint32_t mask);

/* --------------------------------------------------------------- status --- */
int dual_status_clear(uint32_t* status, int device, void* stream);
/* Synchronous read of a device status word (not capturable). */
int dual_status_read(const uint32_t* status, uint32_t* value_out, int device, void* stream);

/* ------------------------------------------------- peer memory / topology ---
 * Replace the ctypes CUDA-IPC helper V/nvlink_cooperation/cuda_ipc.py:18-88
 * (Cuda.allocate/open/close/free/enable_peer/attributes) and the NVLink checks of
 * peer/host4.py:27-62.  Handles are the 64-byte cudaIpcMemHandle_t payload. */
int dual_supplier_alloc(int device, size_t bytes, void** ptr_out, unsigned char handle_out[64]);
int dual_supplier_free(int device, void* ptr);
int dual_ipc_open(int device, const unsigned char handle[64], void** ptr_out);
int dual_ipc_close(int device, void* ptr);
int dual_enable_peer(int device, int peer);
int dual_can_access_peer(int device, int peer, int* out);
/* attr: 0 performance rank, 1 access supported, 2 native atomics (cudaDevP2PAttr*) */
int dual_p2p_attribute(int src, int dst, int attr, int* value);
/* memory_type: cudaMemoryType of ptr; owner_device: its device */
int dual_pointer_info(const void* ptr, int* memory_type, int* owner_device);
int dual_device_count(int* count);

#ifdef __cplusplus
}
#endif

#endif /* DUAL_B200_H */
