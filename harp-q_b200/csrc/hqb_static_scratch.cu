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
// Set-up: the first call on a device, with that device current, resolves the array's
// address on that device with cudaGetSymbolAddress and enqueues a clear of the whole
// array on the caller's stream.  Later calls reuse the cached address.
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
void* g_scratch_on_device[kMaxDevices];  // resolved once per device, never released

// Address of this device's scratch; the first call per device resolves it and clears
// the array on `st`.
cudaError_t device_scratch(int device, cudaStream_t st, void** out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_on_device[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_scratch);
    if (e != cudaSuccess) return e;
    if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255u) != 0) return cudaErrorInvalidDevicePointer;
    e = cudaMemsetAsync(p, 0, HQB_NOALLOC_SCRATCH_BYTES, st);
    if (e != cudaSuccess) return e;
    g_scratch_on_device[device] = p;
  }
  *out = g_scratch_on_device[device];
  return cudaSuccess;
}

}  // namespace

extern "C" HQB_API int hqb_gemv_noalloc(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype,
                                        uint32_t batch, const void* bias, int bias_dtype, void* y, int y_dtype,
                                        void* stream) {
  if (m == nullptr || x == nullptr || y == nullptr) return HQB_ERR_INVALID;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
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
