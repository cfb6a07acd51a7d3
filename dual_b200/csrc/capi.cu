// C ABI entry points (include/dual_b200.h): argument checks, error mapping,
// kernel launches, IPC / peer access / topology helpers.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "dual_b200.h"
#include "decode.cuh"
#include "device_guard.h"
#include "kv_write.cuh"
#include "migrate.cuh"
#include "pack.cuh"
#include "prefill.cuh"
#include "stage.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint32_t> g_inject{0};  // DUAL_INJECT_* bits set by dual_debug_inject (tests only)

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DUAL_ECUDA, "%s: CUDA error %d (%s)", what, int(e), cudaGetErrorString(e));
}

#define DUAL_CHECK_CUDA(expr, what)            \
  do {                                         \
    cudaError_t _e = (expr);                   \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

// Makes `device` current for the rest of the calling entry point and restores the caller's
// current device when it returns (device < 0: the current device).
#define DUAL_USE_DEVICE(device)                                   \
  dual::DeviceGuard device_guard_;                                \
  do {                                                            \
    cudaError_t _e = device_guard_.set(device);                   \
    if (_e != cudaSuccess) return cuda_fail(_e, "cudaSetDevice"); \
  } while (0)

// `device`, or the calling thread's current device when it is negative.
int resolve_device(int device) {
  if (device >= 0) return device;
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return cur;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u; }

}  // namespace

namespace dual {
// Lets other translation units of this library report through dual_last_error().
void set_last_error_message(const char* message) { g_last_error = message ? message : ""; }
}  // namespace dual

extern "C" {

const char* dual_last_error(void) { return g_last_error.c_str(); }
int dual_abi_version(void) { return 200; }

size_t dual_decode_workspace_size(int batch, int num_ctas) {
  if (batch < 0) batch = 0;
  if (num_ctas <= 0) num_ctas = 148;
  return dual::decode_workspace_bytes(batch, num_ctas);
}

int dual_decode_default_ctas(int device) { return dual::decode_default_grid_g(resolve_device(device)); }

int dual_tiered_decode(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_local,
                       const void* v_local, int64_t local_stride_bytes, int64_t local_capacity,
                       const void* const* peer_k, const void* const* peer_v, int num_peers,
                       int64_t peer_stride_bytes, int64_t peer_slots, const int32_t* kv_indptr,
                       const int32_t* unified_indices, int64_t num_indices, int batch, double sm_scale, void* out,
                       int64_t out_stride_token, int64_t out_stride_head, float* lse, void* workspace,
                       size_t workspace_bytes, int num_ctas, int device, void* stream) {
  g_last_error.clear();
  if (batch < 0) return fail(DUAL_EINVAL, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return DUAL_OK;
  if (!q || !k_local || !v_local || !kv_indptr || !unified_indices || !out || !workspace)
    return fail(DUAL_EINVAL, "null pointer argument");
  if (num_peers < 0 || num_peers > dual::kMaxPeers)
    return fail(DUAL_EINVAL, "num_peers must be in [0, %d] (got %d)", dual::kMaxPeers, num_peers);
  if (!aligned16(k_local) || !aligned16(v_local) || (local_stride_bytes & 15) != 0 ||
      local_stride_bytes < dual::kNumKvHeads * dual::kHeadDim * 2)
    return fail(DUAL_EINVAL, "local pool must be 16-byte aligned with a slot stride >= 2048 B, multiple of 16");
  if (local_capacity < 0 || local_capacity > 0xfffffffeLL)
    return fail(DUAL_EINVAL, "local_capacity out of range");
  if ((q_stride_head & 1) || (q_stride_token & 1) || (out_stride_head & 1) || (out_stride_token & 1) ||
      !aligned16(q) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return fail(DUAL_EINVAL, "q/out must be aligned with even element strides");
  if (num_peers > 0) {
    if (!peer_k || !peer_v) return fail(DUAL_EINVAL, "peer pointer arrays are null");
    if ((peer_stride_bytes & 15) != 0 || peer_stride_bytes < dual::kNumKvHeads * dual::kHeadDim * 2 ||
        peer_slots <= 0)
      return fail(DUAL_EINVAL, "peer banks need a 16-byte multiple slot stride >= 2048 B and slots > 0");
    for (int i = 0; i < num_peers; ++i)
      if (!peer_k[i] || !peer_v[i] || !aligned16(peer_k[i]) || !aligned16(peer_v[i]))
        return fail(DUAL_EINVAL, "peer bank %d pointer null or not 16-byte aligned", i);
  }
  if (!(sm_scale > 0.0)) return fail(DUAL_EINVAL, "sm_scale must be positive");
  DUAL_USE_DEVICE(device);
  if (num_ctas <= 0) num_ctas = dual::decode_default_grid_g(resolve_device(device));
  const size_t need = dual::decode_workspace_bytes(batch, num_ctas);
  if (workspace_bytes < need)
    return fail(DUAL_ENOSPACE, "workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(DUAL_EINVAL, "workspace must be 256-byte aligned");

  dual::TieredDecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride_tok = q_stride_token;
  p.q_stride_head = q_stride_head;
  p.k_local = static_cast<const char*>(k_local);
  p.v_local = static_cast<const char*>(v_local);
  p.local_stride = local_stride_bytes;
  p.local_capacity = local_capacity;
  for (int i = 0; i < dual::kMaxPeers; ++i) {
    p.peer_k[i] = i < num_peers ? static_cast<const char*>(peer_k[i]) : nullptr;
    p.peer_v[i] = i < num_peers ? static_cast<const char*>(peer_v[i]) : nullptr;
  }
  p.num_peers = num_peers;
  p.peer_stride = peer_stride_bytes;
  p.peer_slots = peer_slots;
  p.indptr = kv_indptr;
  p.indices = unified_indices;
  p.num_indices = num_indices < 0 ? 0 : num_indices;
  p.batch = batch;
  p.scale_log2 = static_cast<float>(sm_scale * 1.4426950408889634);
  p.status = static_cast<unsigned*>(workspace);
  p.counters = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + 256);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + dual::decode_workspace_head_bytes(batch));
  p.grid_g = num_ctas;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_tok = out_stride_token;
  p.out_stride_head = out_stride_head;
  p.lse = lse;
  cudaError_t e = dual::launch_tiered_decode(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tiered decode launch");
  return DUAL_OK;
}

int dual_decode_workspace_reset(void* workspace, size_t workspace_bytes, int batch, int device, void* stream) {
  g_last_error.clear();
  if (!workspace || batch < 0) return fail(DUAL_EINVAL, "null workspace or negative batch");
  const size_t head = dual::decode_workspace_head_bytes(batch);
  if (workspace_bytes < head) return fail(DUAL_ENOSPACE, "workspace too small: need %zu bytes, got %zu", head,
                                          workspace_bytes);
  DUAL_USE_DEVICE(device);
  DUAL_CHECK_CUDA(cudaMemsetAsync(workspace, 0, head, static_cast<cudaStream_t>(stream)), "workspace reset");
  return DUAL_OK;
}

int dual_append_plan(const int32_t* qo_indptr_host, const int32_t* kv_indptr_host, const int32_t* remote_counts_host,
                     int batch, int causal, int32_t* work_host, int64_t max_work, int64_t* num_work) {
  g_last_error.clear();
  if (batch < 0 || !num_work) return fail(DUAL_EINVAL, "bad append plan arguments");
  if (batch > 0 && (!qo_indptr_host || !kv_indptr_host)) return fail(DUAL_EINVAL, "null indptr");
  for (int b = 0; b < batch; ++b) {
    const int64_t ql = int64_t(qo_indptr_host[b + 1]) - qo_indptr_host[b];
    const int64_t kl = int64_t(kv_indptr_host[b + 1]) - kv_indptr_host[b];
    if (ql < 0 || kl < 0) return fail(DUAL_EINVAL, "request %d: negative length", b);
    if (causal && kl < ql) return fail(DUAL_EINVAL, "request %d: causal append needs kv length >= query length", b);
  }
  if (remote_counts_host)
    for (int b = 0; b < batch; ++b)
      if (remote_counts_host[b] < 0) return fail(DUAL_EINVAL, "request %d: negative remote count", b);
  *num_work = dual::append_plan(qo_indptr_host, kv_indptr_host, remote_counts_host, batch, causal, work_host, max_work);
  return DUAL_OK;
}

int dual_tiered_append(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_local,
                       const void* v_local, int64_t local_stride_bytes, int64_t local_capacity,
                       const void* const* peer_k, const void* const* peer_v, int num_peers,
                       int64_t peer_stride_bytes, int64_t peer_slots, const int32_t* qo_indptr,
                       const int32_t* kv_indptr, const int32_t* unified_indices, int64_t num_indices, int batch,
                       int causal, double sm_scale, const int32_t* work, int64_t num_work, void* out,
                       int64_t out_stride_token, int64_t out_stride_head, float* lse, uint32_t* status, int device,
                       void* stream) {
  g_last_error.clear();
  if (batch < 0 || num_work < 0) return fail(DUAL_EINVAL, "negative batch or work count");
  if (batch == 0 || num_work == 0) return DUAL_OK;
  if (num_work > 0x7fffffffLL) return fail(DUAL_EINVAL, "too many work items");
  if (!q || !k_local || !v_local || !qo_indptr || !kv_indptr || !unified_indices || !work || !out || !status)
    return fail(DUAL_EINVAL, "null pointer argument");
  if (num_peers < 0 || num_peers > dual::kMaxPeers) return fail(DUAL_EINVAL, "num_peers out of range");
  const int64_t min_stride = int64_t(dual::kNumKvHeads) * dual::kHeadDim * 2;
  if (!aligned16(k_local) || !aligned16(v_local) || (local_stride_bytes & 15) || local_stride_bytes < min_stride)
    return fail(DUAL_EINVAL, "local pool must be 16-byte aligned with a slot stride >= 2048 B, multiple of 16");
  if (local_capacity < 0 || local_capacity > 0xfffffffeLL) return fail(DUAL_EINVAL, "local_capacity out of range");
  if ((q_stride_head % 8) || (q_stride_token % 8) || (out_stride_head % 8) || (out_stride_token % 8) ||
      !aligned16(q) || !aligned16(out))
    return fail(DUAL_EINVAL, "q/out must be 16-byte aligned with element strides that are multiples of 8");
  if (num_peers > 0) {
    if (!peer_k || !peer_v) return fail(DUAL_EINVAL, "peer pointer arrays are null");
    if ((peer_stride_bytes & 15) || peer_stride_bytes < min_stride || peer_slots <= 0)
      return fail(DUAL_EINVAL, "peer banks need a 16-byte multiple slot stride >= 2048 B and slots > 0");
    for (int i = 0; i < num_peers; ++i)
      if (!peer_k[i] || !peer_v[i] || !aligned16(peer_k[i]) || !aligned16(peer_v[i]))
        return fail(DUAL_EINVAL, "peer bank %d pointer null or not 16-byte aligned", i);
  }
  if (!(sm_scale > 0.0)) return fail(DUAL_EINVAL, "sm_scale must be positive");
  DUAL_USE_DEVICE(device);
  dual::AppendParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride_tok = q_stride_token;
  p.q_stride_head = q_stride_head;
  p.k_local = static_cast<const char*>(k_local);
  p.v_local = static_cast<const char*>(v_local);
  p.local_stride = local_stride_bytes;
  p.local_capacity = local_capacity;
  for (int i = 0; i < dual::kMaxPeers; ++i) {
    p.peer_k[i] = i < num_peers ? static_cast<const char*>(peer_k[i]) : nullptr;
    p.peer_v[i] = i < num_peers ? static_cast<const char*>(peer_v[i]) : nullptr;
  }
  p.num_peers = num_peers;
  p.peer_stride = peer_stride_bytes;
  p.peer_slots = peer_slots;
  p.qo_indptr = qo_indptr;
  p.kv_indptr = kv_indptr;
  p.indices = unified_indices;
  p.num_indices = num_indices < 0 ? 0 : num_indices;
  p.batch = batch;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(sm_scale * 1.4426950408889634);
  p.work = reinterpret_cast<const int4*>(work);
  p.num_work = int(num_work);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_tok = out_stride_token;
  p.out_stride_head = out_stride_head;
  p.lse = lse;
  p.status = status;
  p.inject = g_inject.load(std::memory_order_relaxed);
  cudaError_t e = dual::launch_tiered_append(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tiered append launch");
  return DUAL_OK;
}

int dual_stage_remote_rows(const void* const* peer_k, const void* const* peer_v, void* const* stage_k,
                           void* const* stage_v, int num_banks, int64_t peer_stride_bytes,
                           int64_t stage_stride_bytes, int64_t bank_slots, int64_t row_bytes,
                           const int32_t* unified_indices, int64_t num_indices, int64_t local_capacity,
                           uint32_t* status, int max_ctas, int device, void* stream) {
  g_last_error.clear();
  if (num_indices < 0) return fail(DUAL_EINVAL, "num_indices must be >= 0");
  if (num_indices == 0) return DUAL_OK;
  if (!unified_indices || !status) return fail(DUAL_EINVAL, "null pointer argument");
  if (num_banks <= 0 || num_banks > dual::kMaxPeers)
    return fail(DUAL_EINVAL, "num_banks must be in [1, %d] (got %d)", dual::kMaxPeers, num_banks);
  if (!peer_k || !peer_v || !stage_k || !stage_v) return fail(DUAL_EINVAL, "bank / stage pointer arrays are null");
  if (row_bytes <= 0 || (row_bytes & 15)) return fail(DUAL_EINVAL, "row_bytes must be a positive multiple of 16");
  if ((peer_stride_bytes & 15) || (stage_stride_bytes & 15) || peer_stride_bytes < row_bytes ||
      stage_stride_bytes < row_bytes)
    return fail(DUAL_EINVAL, "strides must be multiples of 16 bytes and at least row_bytes");
  if (bank_slots <= 0) return fail(DUAL_EINVAL, "bank_slots must be positive");
  if (local_capacity < 0 || local_capacity > 0xfffffffeLL) return fail(DUAL_EINVAL, "local_capacity out of range");
  for (int i = 0; i < num_banks; ++i)
    if (!peer_k[i] || !peer_v[i] || !stage_k[i] || !stage_v[i] || !aligned16(peer_k[i]) || !aligned16(peer_v[i]) ||
        !aligned16(stage_k[i]) || !aligned16(stage_v[i]))
      return fail(DUAL_EINVAL, "bank %d: bank or stage pointer null or not 16-byte aligned", i);
  DUAL_USE_DEVICE(device);
  dual::StageParams p{};
  for (int i = 0; i < dual::kMaxPeers; ++i) {
    p.peer_k[i] = i < num_banks ? static_cast<const char*>(peer_k[i]) : nullptr;
    p.peer_v[i] = i < num_banks ? static_cast<const char*>(peer_v[i]) : nullptr;
    p.stage_k[i] = i < num_banks ? static_cast<char*>(stage_k[i]) : nullptr;
    p.stage_v[i] = i < num_banks ? static_cast<char*>(stage_v[i]) : nullptr;
  }
  p.banks = num_banks;
  p.peer_stride = peer_stride_bytes;
  p.stage_stride = stage_stride_bytes;
  p.bank_slots = bank_slots;
  p.row_bytes = row_bytes;
  p.indices = unified_indices;
  p.n = num_indices;
  p.local_capacity = local_capacity;
  p.status = status;
  cudaError_t e = dual::launch_stage_rows(p, max_ctas, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "stage_remote_rows launch");
  return DUAL_OK;
}

int dual_stage_bank_range(const void* const* peer_k, const void* const* peer_v, void* const* stage_k,
                          void* const* stage_v, int num_banks, int64_t peer_stride_bytes,
                          int64_t stage_stride_bytes, int64_t bank_slots, int64_t row_bytes,
                          const int64_t* row_begin, const int64_t* row_end, void* const* streams, int device) {
  g_last_error.clear();
  if (num_banks <= 0 || num_banks > dual::kMaxPeers)
    return fail(DUAL_EINVAL, "num_banks must be in [1, %d] (got %d)", dual::kMaxPeers, num_banks);
  if (!peer_k || !peer_v || !stage_k || !stage_v || !row_begin || !row_end || !streams)
    return fail(DUAL_EINVAL, "null pointer argument");
  if (row_bytes <= 0 || (row_bytes & 15)) return fail(DUAL_EINVAL, "row_bytes must be a positive multiple of 16");
  if ((peer_stride_bytes & 15) || (stage_stride_bytes & 15) || peer_stride_bytes < row_bytes ||
      stage_stride_bytes < row_bytes)
    return fail(DUAL_EINVAL, "strides must be multiples of 16 bytes and at least row_bytes");
  if (bank_slots <= 0) return fail(DUAL_EINVAL, "bank_slots must be positive");
  for (int i = 0; i < num_banks; ++i) {
    if (!peer_k[i] || !peer_v[i] || !stage_k[i] || !stage_v[i])
      return fail(DUAL_EINVAL, "bank %d: bank or stage pointer is null", i);
    if (row_begin[i] < 0 || row_end[i] > bank_slots || row_begin[i] > row_end[i])
      return fail(DUAL_EINVAL, "bank %d: row range [%lld, %lld) outside [0, %lld]", i, (long long)row_begin[i],
                  (long long)row_end[i], (long long)bank_slots);
  }
  DUAL_USE_DEVICE(device);
  for (int i = 0; i < num_banks; ++i) {
    const int64_t rows = row_end[i] - row_begin[i];
    if (rows == 0) continue;
    cudaStream_t st = static_cast<cudaStream_t>(streams[i]);
    const void* src[2] = {peer_k[i], peer_v[i]};
    void* dst[2] = {stage_k[i], stage_v[i]};
    for (int plane = 0; plane < 2; ++plane) {
      const char* s = static_cast<const char*>(src[plane]) + row_begin[i] * peer_stride_bytes;
      char* d = static_cast<char*>(dst[plane]) + row_begin[i] * stage_stride_bytes;
      cudaError_t e;
      if (peer_stride_bytes == row_bytes && stage_stride_bytes == row_bytes)
        e = cudaMemcpyAsync(d, s, size_t(rows * row_bytes), cudaMemcpyDefault, st);
      else
        e = cudaMemcpy2DAsync(d, size_t(stage_stride_bytes), s, size_t(peer_stride_bytes), size_t(row_bytes),
                              size_t(rows), cudaMemcpyDefault, st);
      if (e != cudaSuccess) return cuda_fail(e, "stage_bank_range copy");
    }
  }
  return DUAL_OK;
}

int dual_pack_read_order(int32_t* tier, int32_t* slot, int64_t table_rows, int64_t table_stride,
                         const int32_t* req_pool_indices,
                         const int32_t* seq_lens, const int32_t* prefix_lens, const int64_t* new_loc, int batch,
                         int64_t local_capacity, int remote_rows, int tile_rows, int32_t* full_out,
                         int32_t* history_out, uint32_t* status, int device, void* stream) {
  g_last_error.clear();
  if (batch < 0) return fail(DUAL_EINVAL, "batch must be >= 0");
  if (batch == 0) return DUAL_OK;
  if (!tier || !slot || !req_pool_indices || !seq_lens || !full_out)
    return fail(DUAL_EINVAL, "null pointer argument");
  if (remote_rows < 0 || (remote_rows > 0 && remote_rows >= tile_rows))
    return fail(DUAL_EINVAL, "need remote_rows == 0 or 0 < remote_rows < tile_rows (got %d/%d)", remote_rows,
                tile_rows);
  if (history_out && !prefix_lens) return fail(DUAL_EINVAL, "history_out requires prefix_lens");
  if (local_capacity < 0 || local_capacity > 0x7ffffffeLL) return fail(DUAL_EINVAL, "local_capacity out of range");
  DUAL_USE_DEVICE(device);
  if (table_rows <= 0 || table_stride <= 0) return fail(DUAL_EINVAL, "empty page tables");
  dual::PackParams p{};
  p.tier = tier;
  p.slot = slot;
  p.rows = table_rows;
  p.stride = table_stride;
  p.req = req_pool_indices;
  p.seq = seq_lens;
  p.prefix = prefix_lens;
  p.new_loc = new_loc;
  p.batch = batch;
  p.local_capacity = local_capacity;
  p.remote_rows = remote_rows;
  p.tile_rows = tile_rows;
  p.full = full_out;
  p.history = history_out;
  p.status = status;
  cudaError_t e = dual::launch_pack_read_order(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pack_read_order launch");
  return DUAL_OK;
}

int dual_write_prefill_layout(int32_t* tier, int32_t* slot, int64_t table_rows, int64_t table_stride,
                              const int32_t* req_pool_indices, const int32_t* start, const int32_t* length,
                              const int32_t* prefix, const void* locations, int loc_is_int64, int batch,
                              int max_length, uint32_t* status, int device, void* stream) {
  g_last_error.clear();
  if (batch < 0 || max_length < 0) return fail(DUAL_EINVAL, "negative batch or max_length");
  if (batch == 0 || max_length == 0) return DUAL_OK;
  if (!tier || !slot || !req_pool_indices || !prefix || !locations) return fail(DUAL_EINVAL, "null pointer argument");
  DUAL_USE_DEVICE(device);
  if (table_rows <= 0 || table_stride <= 0) return fail(DUAL_EINVAL, "empty page tables");
  dual::LayoutParams p{};
  p.tier = tier;
  p.slot = slot;
  p.rows = table_rows;
  p.stride = table_stride;
  p.req = req_pool_indices;
  p.start = start;
  p.length = length;
  p.prefix = prefix;
  p.loc64 = loc_is_int64 ? static_cast<const int64_t*>(locations) : nullptr;
  p.loc32 = loc_is_int64 ? nullptr : static_cast<const int32_t*>(locations);
  p.batch = batch;
  p.status = status;
  cudaError_t e = dual::launch_write_layout(p, max_length, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "write_prefill_layout launch");
  return DUAL_OK;
}

int dual_set_kv_buffer(void* k_local, void* v_local, int64_t local_stride_bytes, int64_t local_capacity,
                       const void* k, int64_t k_stride_token, const void* v, int64_t v_stride_token,
                       const void* locations, int loc_is_int64, int64_t n, uint32_t* status, int device,
                       void* stream) {
  g_last_error.clear();
  if (n < 0) return fail(DUAL_EINVAL, "n must be >= 0");
  if (n == 0) return DUAL_OK;
  if (!k_local || !v_local || !k || !v || !locations || !status) return fail(DUAL_EINVAL, "null pointer argument");
  const int64_t row = int64_t(dual::kNumKvHeads) * dual::kHeadDim * 2;
  if (!aligned16(k_local) || !aligned16(v_local) || (local_stride_bytes & 15) || local_stride_bytes < row)
    return fail(DUAL_EINVAL, "local pools must be 16-byte aligned with a slot stride >= 2048 B, multiple of 16");
  if (!aligned16(k) || !aligned16(v) || (k_stride_token % 8) || (v_stride_token % 8) ||
      k_stride_token < row / 2 || v_stride_token < row / 2)
    return fail(DUAL_EINVAL, "k/v must be 16-byte aligned with token strides >= 1024 elements, multiples of 8");
  if (local_capacity < 0) return fail(DUAL_EINVAL, "local_capacity must be >= 0");
  DUAL_USE_DEVICE(device);
  dual::KvWriteParams p{};
  p.k_local = static_cast<char*>(k_local);
  p.v_local = static_cast<char*>(v_local);
  p.local_stride = local_stride_bytes;
  p.capacity = local_capacity;
  p.k = static_cast<const char*>(k);
  p.v = static_cast<const char*>(v);
  p.k_stride = k_stride_token * 2;
  p.v_stride = v_stride_token * 2;
  p.loc64 = loc_is_int64 ? static_cast<const int64_t*>(locations) : nullptr;
  p.loc32 = loc_is_int64 ? nullptr : static_cast<const int32_t*>(locations);
  p.n = n;
  p.status = status;
  cudaError_t e = dual::launch_set_kv_buffer(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "set_kv_buffer launch");
  return DUAL_OK;
}

int dual_migrate_copy(const int64_t* local_planes, const int64_t* remote_planes, int num_planes, int num_banks,
                      const int64_t* source, const int64_t* target, int64_t n, int reverse, int64_t row_bytes,
                      int64_t local_slots, int64_t remote_slots, uint32_t* status, int max_ctas, int device,
                      void* stream) {
  g_last_error.clear();
  if (n < 0) return fail(DUAL_EINVAL, "n must be >= 0");
  if (n == 0) return DUAL_OK;
  if (!local_planes || !remote_planes || !source || !target || !status)
    return fail(DUAL_EINVAL, "null pointer argument");
  if (num_planes <= 0 || num_banks <= 0) return fail(DUAL_EINVAL, "num_planes and num_banks must be positive");
  if (row_bytes <= 0 || (row_bytes & 15)) return fail(DUAL_EINVAL, "row_bytes must be a positive multiple of 16");
  if (local_slots <= 0 || remote_slots <= 0) return fail(DUAL_EINVAL, "pool sizes must be positive");
  DUAL_USE_DEVICE(device);
  dual::MigrateParams p{};
  p.local_planes = local_planes;
  p.remote_planes = remote_planes;
  p.planes = num_planes;
  p.banks = num_banks;
  p.source = source;
  p.target = target;
  p.n = n;
  p.reverse = reverse ? 1 : 0;
  p.row_bytes = row_bytes;
  p.local_slots = local_slots;
  p.remote_slots = remote_slots;
  p.status = status;
  cudaError_t e = dual::launch_migrate_copy(p, max_ctas, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "migrate_copy launch");
  return DUAL_OK;
}

int dual_debug_inject(uint32_t mask) {
  g_last_error.clear();
  if (mask & ~uint32_t(DUAL_INJECT_APPEND_WITHHOLD_K0)) return fail(DUAL_EINVAL, "unknown injection bits 0x%x", mask);
  g_inject.store(mask, std::memory_order_relaxed);
  return DUAL_OK;
}

int dual_status_clear(uint32_t* status, int device, void* stream) {
  g_last_error.clear();
  if (!status) return fail(DUAL_EINVAL, "null status");
  DUAL_USE_DEVICE(device);
  DUAL_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(uint32_t), static_cast<cudaStream_t>(stream)), "status clear");
  return DUAL_OK;
}

int dual_status_read(const uint32_t* status, uint32_t* value_out, int device, void* stream) {
  g_last_error.clear();
  if (!status || !value_out) return fail(DUAL_EINVAL, "null pointer argument");
  DUAL_USE_DEVICE(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DUAL_CHECK_CUDA(cudaMemcpyAsync(value_out, status, sizeof(uint32_t), cudaMemcpyDeviceToHost, s), "status read");
  DUAL_CHECK_CUDA(cudaStreamSynchronize(s), "status read sync");
  return DUAL_OK;
}

// ------------------------------------------------------------------ IPC / P2P
int dual_supplier_alloc(int device, size_t bytes, void** ptr_out, unsigned char handle_out[64]) {
  g_last_error.clear();
  if (!ptr_out || !handle_out || bytes == 0) return fail(DUAL_EINVAL, "bad supplier_alloc arguments");
  DUAL_USE_DEVICE(device);
  void* ptr = nullptr;
  DUAL_CHECK_CUDA(cudaMalloc(&ptr, bytes), "cudaMalloc (supplier bank)");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    cudaFree(ptr);
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  std::memcpy(handle_out, &h, 64);
  *ptr_out = ptr;
  return DUAL_OK;
}

int dual_supplier_free(int device, void* ptr) {
  g_last_error.clear();
  DUAL_USE_DEVICE(device);
  DUAL_CHECK_CUDA(cudaFree(ptr), "cudaFree (supplier bank)");
  return DUAL_OK;
}

int dual_ipc_open(int device, const unsigned char handle[64], void** ptr_out) {
  g_last_error.clear();
  if (!handle || !ptr_out) return fail(DUAL_EINVAL, "null pointer argument");
  DUAL_USE_DEVICE(device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, 64);
  DUAL_CHECK_CUDA(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return DUAL_OK;
}

int dual_ipc_close(int device, void* ptr) {
  g_last_error.clear();
  DUAL_USE_DEVICE(device);
  DUAL_CHECK_CUDA(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  return DUAL_OK;
}

int dual_can_access_peer(int device, int peer, int* out) {
  g_last_error.clear();
  if (!out) return fail(DUAL_EINVAL, "null out");
  DUAL_CHECK_CUDA(cudaDeviceCanAccessPeer(out, device, peer), "cudaDeviceCanAccessPeer");
  return DUAL_OK;
}

int dual_enable_peer(int device, int peer) {
  g_last_error.clear();
  int can = 0;
  DUAL_CHECK_CUDA(cudaDeviceCanAccessPeer(&can, device, peer), "cudaDeviceCanAccessPeer");
  if (!can) return fail(DUAL_EUNSUPPORTED, "device %d cannot access peer %d", device, peer);
  DUAL_USE_DEVICE(device);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return DUAL_OK;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  return DUAL_OK;
}

int dual_p2p_attribute(int src, int dst, int attr, int* value) {
  g_last_error.clear();
  if (!value) return fail(DUAL_EINVAL, "null value");
  cudaDeviceP2PAttr a;
  switch (attr) {
    case 0: a = cudaDevP2PAttrPerformanceRank; break;
    case 1: a = cudaDevP2PAttrAccessSupported; break;
    case 2: a = cudaDevP2PAttrNativeAtomicSupported; break;
    default: return fail(DUAL_EINVAL, "unknown p2p attribute %d", attr);
  }
  DUAL_CHECK_CUDA(cudaDeviceGetP2PAttribute(value, a, src, dst), "cudaDeviceGetP2PAttribute");
  return DUAL_OK;
}

int dual_pointer_info(const void* ptr, int* memory_type, int* owner_device) {
  g_last_error.clear();
  if (!memory_type || !owner_device) return fail(DUAL_EINVAL, "null out pointers");
  cudaPointerAttributes attr;
  DUAL_CHECK_CUDA(cudaPointerGetAttributes(&attr, ptr), "cudaPointerGetAttributes");
  *memory_type = int(attr.type);
  *owner_device = attr.device;
  return DUAL_OK;
}

int dual_device_count(int* count) {
  g_last_error.clear();
  if (!count) return fail(DUAL_EINVAL, "null count");
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  return DUAL_OK;
}

}  // extern "C"
