// Captured decode steps (hqb_step_*): a list of GEMV calls, optionally with the step's
// host->device input copies and device->host output copies, recorded once as a CUDA graph
// and launched with one call.
//
// Copies between page-locked host memory and the device run as small copy kernels when
// both ends are device-addressable (page-locked host memory is, under unified virtual
// addressing) and 16-byte aligned: launched with programmatic dependent launch, the input
// copy lets the GEMV grid start its weight loads while x is still arriving, and the output
// copy starts as the GEMV grid drains and waits for it before reading y.  Other copies are
// one cudaMemcpyAsync each.
#include <cuda_runtime.h>

#include <cstdint>
#include <new>
#include <vector>

#include "harpq_b200.h"
#include "hqb_device.cuh"
#include "hqb_internal.h"

namespace hqb {
namespace {

constexpr unsigned kCopyThreads = 256;
constexpr unsigned kCopyMaxBlocks = 64;

// dst[i] = src[i] for 16-byte words, grid-stride.  after_gemv: the copy reads the GEMVs'
// outputs, so it waits for the preceding grid; otherwise it lets the following grid start.
__global__ void __launch_bounds__(kCopyThreads) step_copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                                 uint64_t words, int after_gemv) {
  if (after_gemv) griddep_wait();
  else griddep_launch_dependents();
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kCopyThreads;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(kCopyThreads) + threadIdx.x; i < words; i += stride)
    dst[i] = src[i];
}

// The device address of p, or nullptr when the device cannot reach it directly.
const void* device_view(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return p;
  if (a.type == cudaMemoryTypeHost) return a.devicePointer;
  return nullptr;
}

// A copy as the step records it: kernel != 0 when both ends have 16-byte aligned device
// addresses (dst/src then hold those), else the caller's pointers for cudaMemcpyAsync.
struct StepCopy {
  hqb_copy c;
  int kernel;
};

// Resolved before the capture begins (pointer queries are not stream work).
StepCopy resolve_copy(const hqb_copy& c) {
  const void* src = device_view(c.src);
  void* dst = const_cast<void*>(device_view(c.dst));
  const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | c.bytes) & 15u) == 0;
  if (src == nullptr || dst == nullptr || !aligned) return StepCopy{c, 0};
  return StepCopy{hqb_copy{dst, src, c.bytes}, 1};
}

cudaError_t step_copy(const StepCopy& sc, bool after_gemv, cudaStream_t s) {
  const hqb_copy& c = sc.c;
  if (c.bytes == 0) return cudaSuccess;
  if (!sc.kernel) return cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDefault, s);
  void* dst = c.dst;
  const void* src = c.src;
  const uint64_t words = c.bytes / 16;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(
      words / kCopyThreads + 1 < kCopyMaxBlocks ? words / kCopyThreads + 1 : kCopyMaxBlocks));
  cfg.blockDim = dim3(kCopyThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = after_gemv ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, step_copy_kernel, static_cast<uint4*>(dst), static_cast<const uint4*>(src), words,
                            after_gemv ? 1 : 0);
}

}  // namespace
}  // namespace hqb

using namespace hqb;

// A captured decode step: the CUDA graph of a batch of GEMV calls.
struct hqb_step {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

extern "C" {

namespace {
int step_create(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes, hqb_step** step,
                bool grouped, const hqb_copy* h2d = nullptr, uint32_t n_h2d = 0, const hqb_copy* d2h = nullptr,
                uint32_t n_d2h = 0);
}

HQB_API int hqb_step_create(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                            hqb_step** step) {
  return step_create(calls, count, workspace, workspace_bytes, step, false);
}

HQB_API int hqb_step_create_grouped(const hqb_gemv_call* calls, uint32_t count, void* workspace,
                                    uint64_t workspace_bytes, hqb_step** step) {
  return step_create(calls, count, workspace, workspace_bytes, step, true);
}

HQB_API int hqb_step_create_io(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                               const hqb_copy* h2d, uint32_t n_h2d, const hqb_copy* d2h, uint32_t n_d2h, int grouped,
                               hqb_step** step) {
  if ((n_h2d != 0 && h2d == nullptr) || (n_d2h != 0 && d2h == nullptr)) return HQB_ERR_INVALID;
  for (uint32_t i = 0; i < n_h2d; ++i)
    if (h2d[i].dst == nullptr || h2d[i].src == nullptr) return HQB_ERR_INVALID;
  for (uint32_t i = 0; i < n_d2h; ++i)
    if (d2h[i].dst == nullptr || d2h[i].src == nullptr) return HQB_ERR_INVALID;
  return step_create(calls, count, workspace, workspace_bytes, step, grouped != 0, h2d, n_h2d, d2h, n_d2h);
}

}  // extern "C"

namespace {
int step_create(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes, hqb_step** step,
                bool grouped, const hqb_copy* h2d, uint32_t n_h2d, const hqb_copy* d2h, uint32_t n_d2h) {
  if (step == nullptr || calls == nullptr || count == 0) return HQB_ERR_INVALID;
  *step = nullptr;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return e;
  hqb_step* st = new (std::nothrow) hqb_step();
  if (st == nullptr) {
    cudaStreamDestroy(s);
    return cudaErrorMemoryAllocation;
  }
  std::vector<StepCopy> in, out;
  try {
    for (uint32_t i = 0; i < n_h2d; ++i) in.push_back(resolve_copy(h2d[i]));
    for (uint32_t i = 0; i < n_d2h; ++i) out.push_back(resolve_copy(d2h[i]));
  } catch (...) {
    delete st;
    cudaStreamDestroy(s);
    return cudaErrorMemoryAllocation;
  }
  int status = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (status == cudaSuccess) {
    // the step's input copies, its GEMVs, its output copies (step_copy)
    for (uint32_t i = 0; i < n_h2d && status == cudaSuccess; ++i) status = step_copy(in[i], false, s);
    if (status == cudaSuccess)
      status = grouped ? hqb_gemv_grouped(calls, count, workspace, workspace_bytes, s)
                       : hqb_gemv_batch(calls, count, workspace, workspace_bytes, s);
    for (uint32_t i = 0; i < n_d2h && status == cudaSuccess; ++i) status = step_copy(out[i], true, s);
    cudaGraph_t g = nullptr;
    const cudaError_t end = cudaStreamEndCapture(s, &g);  // always end the capture
    if (status == HQB_OK) status = end;
    st->graph = g;
    if (status == HQB_OK) status = cudaGraphInstantiate(&st->exec, g, 0);
  }
  cudaStreamDestroy(s);
  if (status != HQB_OK) {
    if (st->exec != nullptr) cudaGraphExecDestroy(st->exec);
    if (st->graph != nullptr) cudaGraphDestroy(st->graph);
    delete st;
    cudaGetLastError();
    return status;
  }
  *step = st;
  return HQB_OK;
}
}  // namespace

extern "C" {

HQB_API int hqb_step_launch(hqb_step* step, void* stream) {
  if (step == nullptr || step->exec == nullptr) return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  return cudaGraphLaunch(step->exec, as_stream(stream));
}

HQB_API int hqb_step_destroy(hqb_step* step) {
  if (step == nullptr) return HQB_ERR_INVALID;
  if (step->exec != nullptr) cudaGraphExecDestroy(step->exec);
  if (step->graph != nullptr) cudaGraphDestroy(step->graph);
  delete step;
  return HQB_OK;
}

}  // extern "C"
