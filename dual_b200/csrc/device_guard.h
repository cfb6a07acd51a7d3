// Per-call device selection for the C ABI.
//
// Every entry point takes a device index and launches on a stream of that device, so it has to
// make the device current; the calling thread's current device is the caller's state, though, and
// a call on device 1 from a thread that works on device 0 must leave it on device 0.  DeviceGuard
// makes the device current for the duration of one call and gives the caller's device back when it
// goes out of scope.  The old device is made current again only if its primary context is already
// active: a thread that never used CUDA reports device 0, and switching back to it would create a
// context (and take memory) on a GPU the process may not use at all.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace dual {

namespace detail {
using PrimaryCtxGetStateFn = CUresult (*)(CUdevice, unsigned int*, int*);
using DeviceGetFn = CUresult (*)(CUdevice*, int);

// True if `ordinal`'s primary context is active; true as well when the driver entry points cannot
// be found (then restoring is the safe default).
inline bool primary_context_active(int ordinal) {
  static PrimaryCtxGetStateFn get_state = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuDevicePrimaryCtxGetState", &fn, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return PrimaryCtxGetStateFn(nullptr);
    return reinterpret_cast<PrimaryCtxGetStateFn>(fn);
  }();
  static DeviceGetFn device_get = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuDeviceGet", &fn, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return DeviceGetFn(nullptr);
    return reinterpret_cast<DeviceGetFn>(fn);
  }();
  if (get_state == nullptr || device_get == nullptr) return true;
  CUdevice dev = 0;
  if (device_get(&dev, ordinal) != CUDA_SUCCESS) return true;
  unsigned int flags = 0;
  int active = 0;
  if (get_state(dev, &flags, &active) != CUDA_SUCCESS) return true;
  return active != 0;
}
}  // namespace detail

class DeviceGuard {
 public:
  DeviceGuard() = default;
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
  ~DeviceGuard() {
    if (changed_ && detail::primary_context_active(prev_)) cudaSetDevice(prev_);
  }

  // Makes `device` current (a negative index keeps the current device).  Returns cudaSuccess or
  // the error of cudaGetDevice / cudaSetDevice; on error nothing was changed.
  // Called again, it switches on and still restores the device current before the first call.
  cudaError_t set(int device) {
    if (device < 0) return cudaSuccess;
    int cur = 0;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return e;
    if (cur == device) return cudaSuccess;
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return e;
    if (!changed_) {
      prev_ = cur;
      changed_ = true;
    }
    return cudaSuccess;
  }

 private:
  int prev_ = 0;
  bool changed_ = false;
};

}  // namespace dual
