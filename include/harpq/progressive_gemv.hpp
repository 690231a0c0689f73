// Fused progressive GEMV — the reference's native API
// (reference native/include/harpq/progressive_gemv.hpp:11-75), same types and
// signatures.  LaunchProgressiveGemv runs the B200 kernels behind the C ABI in
// harpq_b200.h; matrices kept resident in the plane layout (harpq_b200.h,
// hqb_gemv*) are the fast path for repeated decode steps.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime_api.h>

#include "harpq/native/stage_codec.hpp"

namespace harpq::native_runtime {

// Geometry copied by value into a launch.  Scales follow the stage-codec layout
// [tile-grid-row, tile-grid-column, row-in-tile, group].
struct ProgressiveGemvGeometry {
  std::uint64_t original_rows = 0;
  std::uint64_t original_columns = 0;
  std::uint64_t padded_rows = 0;
  std::uint64_t padded_columns = 0;
  std::uint64_t tile_rows = 0;
  std::uint64_t tile_columns = 0;
  std::uint64_t group_size = 0;
};

// Device pointers; scale_fp16_bits holds raw IEEE binary16 bit patterns.
struct ProgressiveGemvStageDeviceView {
  const std::uint8_t* packed_codes = nullptr;
  std::uint64_t packed_code_bytes = 0;
  const std::uint16_t* scale_fp16_bits = nullptr;
  std::uint64_t scale_count = 0;
};

struct ProgressiveGemvDeviceView {
  ProgressiveGemvGeometry geometry{};
  ProgressiveGemvStageDeviceView stages[kMaximumStageCount]{};
  std::size_t stage_count = 0;
};

struct ProgressiveGemvIoDeviceView {
  const float* input = nullptr;
  std::uint64_t input_count = 0;
  const float* bias = nullptr;
  std::uint64_t bias_count = 0;
  float* output = nullptr;
  std::uint64_t output_count = 0;
};

// Enqueues a batch-one progressive GEMV on `stream`.  All pointers are device
// pointers that stay valid until the work completes.  Prefix zero writes bias or
// exact zeros.  Returns cudaErrorInvalidValue for an invalid view (nothing is
// enqueued), a pending sticky CUDA error without launching, else the launch status.
// The caller owns synchronisation and asynchronous error handling.
[[nodiscard]] cudaError_t LaunchProgressiveGemv(const ProgressiveGemvIoDeviceView& io,
                                                const ProgressiveGemvDeviceView& matrix,
                                                std::size_t prefix, cudaStream_t stream) noexcept;

// Owning, synchronous wrapper for tests and bring-up: validates the host matrix
// (scales must be exactly FP16-representable), uploads, launches, downloads.
// Throws std::invalid_argument, std::overflow_error or std::runtime_error.
[[nodiscard]] std::vector<float> ProgressiveGemvCuda(const std::vector<float>& input,
                                                     const ProgressiveMatrix& matrix, std::size_t prefix,
                                                     const std::vector<float>& bias = {});

}  // namespace harpq::native_runtime
