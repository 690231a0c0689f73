// Progressive-matrix container and stage-payload codec — the reference's native API
// (reference native/include/harpq/native/stage_codec.hpp:10-72), kept name-for-name so
// existing callers and tests compile unchanged against this library.
//
// DecodeStagePayload and Crc32c parse bytes on the host.  DequantizeStage,
// DequantizePrefix and ProgressiveLinearReference keep their exact results
// (bit-identical FP32): they run on the CUDA device when one is usable and as host
// loops of the same FP32 operations otherwise, so CPU-only callers keep them.
#ifndef HARPQ_B200_NATIVE_STAGE_CODEC_HPP_
#define HARPQ_B200_NATIVE_STAGE_CODEC_HPP_

#include <array>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <vector>

namespace harpq::native_runtime {

inline constexpr std::uint16_t kStageCodecVersion = 1;
inline constexpr std::size_t kMaximumStageCount = 4;

// [tile_grid_rows, tile_grid_columns, tile_rows, groups_per_tile]
using ScaleShape = std::array<std::size_t, 4>;

struct MatrixGeometry {
  std::size_t original_rows;
  std::size_t original_columns;
  std::size_t padded_rows;
  std::size_t padded_columns;
  std::size_t tile_rows;
  std::size_t tile_columns;
  std::size_t group_size;
};

struct DecodedStage {
  std::uint16_t stage_index;
  std::vector<std::uint8_t> packed_codes;  // row-major over the padded matrix, 4 codes/byte
  std::vector<float> scales;               // FP16-decoded, ScaleShape order
  ScaleShape scale_shape;
};

struct ProgressiveMatrix {
  MatrixGeometry geometry;
  std::vector<DecodedStage> stages;  // a contiguous prefix: stages[i].stage_index == i
};

class StageCodecError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

// Parses one "HQSTAGE\0" v1 payload (header, codes, little-endian FP16 scales).
[[nodiscard]] DecodedStage DecodeStagePayload(const std::vector<std::uint8_t>& payload,
                                              std::uint16_t expected_stage,
                                              const ScaleShape& scale_shape);

// One stage decoded to FP32 (original shape, row-major): code * scale, exact.
[[nodiscard]] std::vector<float> DequantizeStage(const ProgressiveMatrix& matrix, std::size_t stage_index);

// Stages [0, prefix) summed in stage order into 0.0f — the bit-exact decoded weight.
[[nodiscard]] std::vector<float> DequantizePrefix(const ProgressiveMatrix& matrix, std::size_t prefix);

// inputs [batch_size][original_columns] -> outputs [batch_size][original_rows], stage-major
// scalar FP32 order with bias added last.
[[nodiscard]] std::vector<float> ProgressiveLinearReference(const std::vector<float>& inputs,
                                                            std::size_t batch_size,
                                                            const ProgressiveMatrix& matrix,
                                                            std::size_t prefix,
                                                            const std::vector<float>& bias = {});

[[nodiscard]] std::uint32_t Crc32c(const std::uint8_t* data, std::size_t size, std::uint32_t crc = 0);

[[nodiscard]] inline std::uint32_t Crc32c(const std::vector<std::uint8_t>& data, std::uint32_t crc = 0) {
  return Crc32c(data.data(), data.size(), crc);
}

}  // namespace harpq::native_runtime

#endif  // HARPQ_B200_NATIVE_STAGE_CODEC_HPP_
