// TEST INFRASTRUCTURE ONLY — C shim over the reference's own fused GEMV kernel.
//
// oracle/build.py compiles this file with the reference's unmodified
// native/src/progressive_gemv.cu (read in place from the reference checkout)
// for sm_100a into oracle/_ref/libharpq_ref_gpu.so.  bench.py uses it to time the
// reference's ProgressiveGemvKernel on the same B200, the same inputs and the
// same weight rotation as the product kernel.  All reference symbols are hidden;
// only hqr_gpu_* are exported.
#include "harpq/progressive_gemv.hpp"

#include <cstdint>

namespace nr = harpq::native_runtime;

#define HQR_API extern "C" __attribute__((visibility("default")))

// geometry: 7 values as in ProgressiveGemvGeometry.  codes/scales: stage_count
// device pointers.  Returns the cudaError_t of LaunchProgressiveGemv.
HQR_API int hqr_gpu_launch(const std::uint64_t* geometry, const void* const* codes,
                           const void* const* scales, std::uint32_t stage_count,
                           std::uint32_t prefix, const float* input, const float* bias,
                           float* output, void* stream) {
  nr::ProgressiveGemvDeviceView view{};
  view.geometry = {geometry[0], geometry[1], geometry[2], geometry[3],
                   geometry[4], geometry[5], geometry[6]};
  const std::uint64_t padded = geometry[2] * geometry[3];
  const std::uint64_t scale_count =
      (geometry[2] / geometry[4]) * (geometry[3] / geometry[5]) * geometry[4] *
      (geometry[5] / geometry[6]);
  for (std::uint32_t s = 0; s < stage_count; ++s) {
    view.stages[s] = {static_cast<const std::uint8_t*>(codes[s]), (padded + 3) / 4,
                      static_cast<const std::uint16_t*>(scales[s]), scale_count};
  }
  view.stage_count = stage_count;
  const nr::ProgressiveGemvIoDeviceView io{
      input, geometry[1], bias, bias != nullptr ? geometry[0] : 0, output, geometry[0]};
  return static_cast<int>(
      nr::LaunchProgressiveGemv(io, view, prefix, static_cast<cudaStream_t>(stream)));
}
