// hqb_gemv_noalloc: the plane-layout GEMV with its scratch in a fixed device array
// that is part of this library's image, so the call itself allocates nothing.
//
// Who needs it: a caller that holds no device allocator (an FFI host that binds only
// this library and has no way to obtain device memory of its own) and a decode step
// that must not allocate, because cudaMalloc and cudaFree synchronize the whole device
// and can fail once weights and caches have claimed the HBM.  Such a caller still gets
// the same kernels as hqb_gemv.
//
// Scratch contents (the layout hqb_gemv uses for a caller workspace):
//   error word (HQB_DEVERR_* bits that kernels OR in), split-row arrival counters and
//       split-row partial sums: must start at zero.  Counters and partial sums return
//       to zero at the end of every call.
//   prepared activations: each call writes them before it reads them, so they need no
//       initial value.
//
// Set-up: every call, with the device current, resolves the array's address on that
// device with cudaGetSymbolAddress; the first call (and a call that finds the address
// changed, after cudaDeviceReset) enqueues a clear of the whole array on the caller's
// stream.  Make the first call before any stream capture.
//
// Recovery: hqb_gemv_noalloc_flags reads (and optionally clears) the error word;
// hqb_gemv_noalloc_reset clears the whole array again, for use after a non-zero word.
//
// Concurrency: there is ONE scratch per device.  Calls whose GPU work overlaps (on
// different streams, or from several host threads without ordering between their
// streams) race on it and give wrong results.  Callers order them (one stream, or
// events).
#include <cuda_runtime.h>

#include <mutex>

#include "harpq_b200.h"
#include "hqb_internal.h"

namespace {

// One copy per device, loaded with the library's device code.  256-byte alignment is
// what hqb_gemv requires of a workspace.
__device__ __align__(256) unsigned char g_gemv_scratch[HQB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_on_device[kMaxDevices];  // last address seen per device (cleared there)

// Address of this device's scratch.  It is resolved on every call (cudaGetSymbolAddress
// allocates nothing): the first call per device, and any call that finds the address
// changed (the module loaded again after cudaDeviceReset), clears the array on `st`.
cudaError_t device_scratch(int device, cudaStream_t st, void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_scratch);
  if (e != cudaSuccess) return e;
  if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255u) != 0) return cudaErrorInvalidDevicePointer;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_on_device[device] != p) {
    e = cudaMemsetAsync(p, 0, HQB_NOALLOC_SCRATCH_BYTES, st);
    if (e != cudaSuccess) return e;
    g_scratch_on_device[device] = p;
  }
  *out = p;
  return cudaSuccess;
}

cudaError_t current_device(int* device) {
  cudaError_t e = cudaGetDevice(device);
  if (e != cudaSuccess) return e;
  if (*device < 0 || *device >= kMaxDevices) return cudaErrorInvalidDevice;
  return cudaSuccess;
}

}  // namespace

extern "C" HQB_API int hqb_gemv_noalloc(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype,
                                        uint32_t batch, const void* bias, int bias_dtype, void* y, int y_dtype,
                                        void* stream) {
  if (m == nullptr || x == nullptr || y == nullptr) return HQB_ERR_INVALID;
  int device = 0;
  cudaError_t e = current_device(&device);
  if (e != cudaSuccess) return e;
  // Same size rule as a caller workspace; 0 means the matrix, batch or dtype is invalid.
  const uint64_t need = hqb_workspace_bytes(m, batch, x_dtype, device);
  if (need == 0) return HQB_ERR_INVALID;
  if (need > HQB_NOALLOC_SCRATCH_BYTES) return HQB_ERR_SCRATCH_LIMIT;
  const cudaError_t prior = hqb::take_prior_error();
  if (prior != cudaSuccess) return prior;
  void* scratch = nullptr;
  e = device_scratch(device, hqb::as_stream(stream), &scratch);
  if (e != cudaSuccess) return e;
  return hqb_gemv(m, prefix, x, x_dtype, batch, bias, bias_dtype, y, y_dtype, scratch, HQB_NOALLOC_SCRATCH_BYTES,
                  stream);
}

// The error word is the scratch's first 4 bytes (the workspace layout of hqb_gemv).
extern "C" HQB_API int hqb_gemv_noalloc_flags(int* host_flags, int clear, void* stream) {
  if (host_flags == nullptr) return HQB_ERR_INVALID;
  int device = 0;
  cudaError_t e = current_device(&device);
  if (e != cudaSuccess) return e;
  void* scratch = nullptr;
  e = device_scratch(device, hqb::as_stream(stream), &scratch);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyAsync(host_flags, scratch, sizeof(int), cudaMemcpyDeviceToHost, hqb::as_stream(stream));
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(scratch, 0, sizeof(int), hqb::as_stream(stream));
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(hqb::as_stream(stream));
}

extern "C" HQB_API int hqb_gemv_noalloc_reset(void* stream) {
  int device = 0;
  cudaError_t e = current_device(&device);
  if (e != cudaSuccess) return e;
  void* scratch = nullptr;
  e = device_scratch(device, hqb::as_stream(stream), &scratch);
  if (e != cudaSuccess) return e;
  return cudaMemsetAsync(scratch, 0, HQB_NOALLOC_SCRATCH_BYTES, hqb::as_stream(stream));
}

extern "C" HQB_API int hqb_gemv_noalloc_scratch(void** ptr) {
  if (ptr == nullptr) return HQB_ERR_INVALID;
  int device = 0;
  cudaError_t e = current_device(&device);
  if (e != cudaSuccess) return e;
  return device_scratch(device, nullptr, ptr);
}
