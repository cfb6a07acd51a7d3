// Allocation-free variant of dual_tiered_decode.
//
// Who needs it: callers that cannot call cudaMalloc or hand this library a
// scratch buffer.  Typical cases are a serving process whose memory manager
// has already reserved nearly all of HBM for its own KV pools and forbids
// out-of-band device allocations (and cudaMalloc would also synchronise the
// device in the middle of a decode loop), or a foreign-language binding that
// can pass the attention tensors it owns but has no way to allocate device
// memory itself.  For them the split-KV partial states live in one fixed
// file-scope __device__ array instead of a caller workspace.
//
// Costs and rules:
//   * every GPU that loads this library holds kNoAllocScratchBytes (8 MiB) of
//     device memory for this array until the process exits;
//   * the array is shared by every call on a device and keeps the last call's
//     contents; calls whose work overlaps on the GPU (e.g. on two streams at
//     once) race on it and must be ordered by the caller;
//   * the first call on each device looks the array's device address up
//     (cudaGetSymbolAddress with that device current) and caches it; make that
//     first call before any stream capture on the device;
//   * sizes beyond the array are rejected: (num_ctas + batch) segments of
//     32 q heads x 132 floats, plus a 256-byte header and batch x 8 arrival
//     counters (rounded up to 256 bytes), must fit in 8 MiB;
//   * every call clears the arrival counters before its kernel, so a call
//     never depends on what an earlier one left in the array;
//   * with status == NULL the kernels record their status bits (bad page ids,
//     timed-out waits) in the array's own header word, which each such call
//     clears first; dual_decode_noalloc_status reads it back, and it is only
//     meaningful until the next call on the device.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "dual_b200.h"
#include "decode.cuh"
#include "device_guard.h"

namespace dual {
void set_last_error_message(const char* message);  // capi.cu
}

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

// Scratch of the allocation-free decode: [status word: 256 B][arrival counters][partials].
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

int noalloc_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  dual::set_last_error_message(buf);  // reported by dual_last_error()
  return code;
}

// `device`, or the calling thread's current device when it is negative (as for dual_tiered_decode).
int resolve_device(int device, int* out) {
  if (device < 0) {
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  }
  if (device >= kMaxDevices) return noalloc_fail(DUAL_EINVAL, "device index %d out of range", device);
  *out = device;
  return DUAL_OK;
}

// Device address of g_decode_scratch on `device` (looked up once per device,
// with that device current; the caller's current device is restored).  In host
// code the symbol itself is only a host stand-in and must never be handed to a
// kernel.
int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[device] == nullptr) {
    dual::DeviceGuard guard;
    cudaError_t e = guard.set(device);
    if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return noalloc_fail(DUAL_ECUDA, "cudaGetSymbolAddress(decode scratch) on device %d: %s", device,
                          cudaGetErrorString(e));
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return DUAL_OK;
}

}  // namespace

extern "C" int dual_tiered_decode_noalloc(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                          const void* k_local, const void* v_local, int64_t local_stride_bytes,
                                          int64_t local_capacity, const void* const* peer_k,
                                          const void* const* peer_v, int num_peers, int64_t peer_stride_bytes,
                                          int64_t peer_slots, const int32_t* kv_indptr,
                                          const int32_t* unified_indices, int64_t num_indices, int batch,
                                          double sm_scale, void* out, int64_t out_stride_token,
                                          int64_t out_stride_head, float* lse, uint32_t* status, int num_ctas,
                                          int device, void* stream) {
  dual::set_last_error_message("");
  if (batch < 0) return noalloc_fail(DUAL_EINVAL, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return DUAL_OK;
  if (!q || !k_local || !v_local || !kv_indptr || !unified_indices || !out)
    return noalloc_fail(DUAL_EINVAL, "null pointer argument");
  if (num_peers < 0 || num_peers > dual::kMaxPeers)
    return noalloc_fail(DUAL_EINVAL, "num_peers must be in [0, %d] (got %d)", dual::kMaxPeers, num_peers);
  const int64_t min_stride = int64_t(dual::kNumKvHeads) * dual::kHeadDim * 2;
  auto aligned16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0u; };
  if (!aligned16(k_local) || !aligned16(v_local) || (local_stride_bytes & 15) != 0 || local_stride_bytes < min_stride)
    return noalloc_fail(DUAL_EINVAL, "local pool must be 16-byte aligned with a slot stride >= 2048 B, multiple of 16");
  if (local_capacity < 0 || local_capacity > 0xfffffffeLL) return noalloc_fail(DUAL_EINVAL, "local_capacity out of range");
  if ((q_stride_head & 1) || (q_stride_token & 1) || (out_stride_head & 1) || (out_stride_token & 1) ||
      !aligned16(q) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return noalloc_fail(DUAL_EINVAL, "q/out must be aligned with even element strides");
  if (num_peers > 0) {
    if (!peer_k || !peer_v) return noalloc_fail(DUAL_EINVAL, "peer pointer arrays are null");
    if ((peer_stride_bytes & 15) != 0 || peer_stride_bytes < min_stride || peer_slots <= 0)
      return noalloc_fail(DUAL_EINVAL, "peer banks need a 16-byte multiple slot stride >= 2048 B and slots > 0");
    for (int i = 0; i < num_peers; ++i)
      if (!peer_k[i] || !peer_v[i] || !aligned16(peer_k[i]) || !aligned16(peer_v[i]))
        return noalloc_fail(DUAL_EINVAL, "peer bank %d pointer null or not 16-byte aligned", i);
  }
  if (!(sm_scale > 0.0)) return noalloc_fail(DUAL_EINVAL, "sm_scale must be positive");
  if (int rc = resolve_device(device, &device)) return rc;
  if (num_ctas <= 0) num_ctas = dual::decode_default_grid_g(device);
  const size_t need = dual::decode_workspace_bytes(batch, num_ctas);
  if (need > kNoAllocScratchBytes)
    return noalloc_fail(DUAL_ENOSPACE,
                        "batch %d with %d CTAs needs %zu bytes of scratch; the allocation-free entry point holds "
                        "%zu (num_ctas + batch <= %zu)",
                        batch, num_ctas, need, kNoAllocScratchBytes,
                        (kNoAllocScratchBytes - dual::decode_workspace_head_bytes(batch)) /
                            (sizeof(float) * dual::DecodeCfg::ROWS * dual::kPartialStride));
  void* scratch = nullptr;
  if (int rc = scratch_address(device, &scratch)) return rc;
  dual::DeviceGuard guard;
  cudaError_t e = guard.set(device);
  if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* status_word = reinterpret_cast<unsigned*>(status);
  if (status_word == nullptr) {
    // The array keeps the previous call's status bits: start this call from zero.
    status_word = static_cast<unsigned*>(scratch);
    e = cudaMemsetAsync(status_word, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "status clear: %s", cudaGetErrorString(e));
  }
  // Arrival counters start at zero in every call (an earlier call that gave up on a wait may have
  // left some behind).
  unsigned* counters = reinterpret_cast<unsigned*>(static_cast<char*>(scratch) + 256);
  e = cudaMemsetAsync(counters, 0, dual::decode_counter_bytes(batch), s);
  if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "counter clear: %s", cudaGetErrorString(e));

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
  p.status = status_word;
  p.counters = counters;
  p.partial = reinterpret_cast<float*>(static_cast<char*>(scratch) + dual::decode_workspace_head_bytes(batch));
  p.grid_g = num_ctas;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_tok = out_stride_token;
  p.out_stride_head = out_stride_head;
  p.lse = lse;
  e = dual::launch_tiered_decode(p, s);
  if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "tiered decode launch: %s", cudaGetErrorString(e));
  return DUAL_OK;
}

extern "C" int dual_decode_noalloc_status(uint32_t* value_out, int device, void* stream) {
  dual::set_last_error_message("");
  if (value_out == nullptr) return noalloc_fail(DUAL_EINVAL, "null value_out");
  if (int rc = resolve_device(device, &device)) return rc;
  void* scratch = nullptr;
  if (int rc = scratch_address(device, &scratch)) return rc;
  dual::DeviceGuard guard;
  cudaError_t e = guard.set(device);
  if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemcpyAsync(value_out, scratch, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return noalloc_fail(DUAL_ECUDA, "status read: %s", cudaGetErrorString(e));
  return DUAL_OK;
}
