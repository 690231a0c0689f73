// CUDA materialize-then-matvec oracle — the reference's native API
// (reference native/include/harpq/cuda_oracle.hpp:9-28), same signatures.
#pragma once

#include <cstddef>
#include <string>
#include <vector>

#include "harpq/native/stage_codec.hpp"

namespace harpq::native_runtime {

// Real CUDA runtime probe; on failure *reason (when non-null) explains why.
[[nodiscard]] bool CudaDeviceAvailable(std::string* reason = nullptr) noexcept;

// Decodes the selected prefix into an FP32 weight matrix on the device (stage order,
// from zero) and evaluates inputs · Wᵀ with deterministic pedantic cuBLAS SGEMM;
// bias, when given, is added once.  Prefix zero is an all-zero matrix; batch zero
// returns an empty vector.  Throws std::invalid_argument / std::overflow_error /
// std::runtime_error.
[[nodiscard]] std::vector<float> ProgressiveLinearCudaOracle(const std::vector<float>& inputs,
                                                             std::size_t batch_size,
                                                             const ProgressiveMatrix& matrix, std::size_t prefix,
                                                             const std::vector<float>& bias = {});

}  // namespace harpq::native_runtime
