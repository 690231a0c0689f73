// C++17 API of the reference (harpq::native_runtime) implemented over this library's
// C ABI.  Validation order, messages' meaning and exception types follow the
// reference so its callers and tests behave the same; the arithmetic runs on the
// device through the sm_100a kernels (the reference's three host functions fall back
// to host loops of the same operations when no device is usable).
//
//   stage codec    reference native/src/stage_codec.cpp:80-339
//   fused GEMV     reference native/src/progressive_gemv.cu:73-541
//   CUDA oracle    reference native/src/cuda_oracle.cu:173-478
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "harpq/cuda_oracle.hpp"
#include "harpq/native/stage_codec.hpp"
#include "harpq/progressive_gemv.hpp"
#include "harpq_b200.h"

namespace harpq::native_runtime {
namespace {

static_assert(sizeof(ProgressiveGemvGeometry) == sizeof(hqb_geometry), "geometry layout");
static_assert(sizeof(ProgressiveGemvStageDeviceView) == sizeof(hqb_raw_stage), "stage view layout");

template <typename Error>
std::size_t Mul(std::size_t a, std::size_t b, const char* what) {
  if (a != 0 && b > std::numeric_limits<std::size_t>::max() / a) throw Error(std::string(what) + " does not fit in size_t");
  return a * b;
}

std::size_t CeilDiv(std::size_t a, std::size_t b) { return a / b + (a % b != 0 ? 1U : 0U); }

[[noreturn]] void ThrowCuda(cudaError_t e, const char* what) {
  std::ostringstream m;
  m << what << " failed: " << cudaGetErrorName(e) << " (" << cudaGetErrorString(e) << ')';
  throw std::runtime_error(m.str());
}

void Check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) ThrowCuda(e, what);
}

void Check(int status, const char* what) { Check(static_cast<cudaError_t>(status), what); }

template <typename T>
class DeviceArray {
 public:
  DeviceArray() = default;
  explicit DeviceArray(std::size_t n) : n_(n) {
    if (n_ != 0) Check(cudaMalloc(reinterpret_cast<void**>(&p_), Mul<std::overflow_error>(n_, sizeof(T), "device allocation")), "cudaMalloc");
  }
  DeviceArray(const DeviceArray&) = delete;
  DeviceArray& operator=(const DeviceArray&) = delete;
  DeviceArray(DeviceArray&& o) noexcept : p_(std::exchange(o.p_, nullptr)), n_(std::exchange(o.n_, 0)) {}
  DeviceArray& operator=(DeviceArray&& o) noexcept {
    if (this != &o) {
      if (p_) static_cast<void>(cudaFree(p_));
      p_ = std::exchange(o.p_, nullptr);
      n_ = std::exchange(o.n_, 0);
    }
    return *this;
  }
  ~DeviceArray() {
    if (p_) static_cast<void>(cudaFree(p_));
  }
  T* get() const noexcept { return p_; }
  std::size_t size() const noexcept { return n_; }

 private:
  T* p_ = nullptr;
  std::size_t n_ = 0;
};

// A non-blocking stream that finishes its queued work before it (and, because it is
// declared after them, the buffers that work uses) goes away.
class Stream {
 public:
  Stream() { Check(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking), "cudaStreamCreateWithFlags"); }
  ~Stream() {
    if (s_) {
      static_cast<void>(cudaStreamSynchronize(s_));
      static_cast<void>(cudaStreamDestroy(s_));
    }
  }
  Stream(const Stream&) = delete;
  Stream& operator=(const Stream&) = delete;
  cudaStream_t get() const noexcept { return s_; }

 private:
  cudaStream_t s_ = nullptr;
};

template <typename T>
void Upload(DeviceArray<T>& dst, const std::vector<T>& src, cudaStream_t s, const char* what) {
  if (!src.empty()) Check(cudaMemcpyAsync(dst.get(), src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice, s), what);
}

hqb_geometry ToGeometry(const MatrixGeometry& g) {
  return hqb_geometry{g.original_rows, g.original_columns, g.padded_rows, g.padded_columns,
                      g.tile_rows,     g.tile_columns,     g.group_size};
}

// Device copy of a host matrix's codes and FP32 scales for stages [0, count).
struct DeviceStagesF32 {
  std::vector<DeviceArray<std::uint8_t>> codes;
  std::vector<DeviceArray<float>> scales;
  std::vector<hqb_raw_stage_f32> views;

  DeviceStagesF32(const ProgressiveMatrix& m, std::size_t count, cudaStream_t s) {
    for (std::size_t i = 0; i < count; ++i) {
      const DecodedStage& st = m.stages[i];
      codes.emplace_back(st.packed_codes.size());
      scales.emplace_back(st.scales.size());
      Upload(codes.back(), st.packed_codes, s, "cudaMemcpyAsync(stage codes H2D)");
      Upload(scales.back(), st.scales, s, "cudaMemcpyAsync(stage scales H2D)");
    }
    for (std::size_t i = 0; i < count; ++i)
      views.push_back(hqb_raw_stage_f32{codes[i].get(), m.stages[i].packed_codes.size(), scales[i].get(),
                                        m.stages[i].scales.size()});
    // The C ABI wants one entry per resident stage; entries past `count` are unused.
    while (views.size() < std::max<std::size_t>(1, m.stages.size())) views.push_back(hqb_raw_stage_f32{});
  }
};

// ---- stage codec ---------------------------------------------------------------------

std::uint16_t Le16(const std::uint8_t* p) { return static_cast<std::uint16_t>(p[0] | (p[1] << 8)); }
std::uint32_t Le32(const std::uint8_t* p) {
  return static_cast<std::uint32_t>(p[0]) | (static_cast<std::uint32_t>(p[1]) << 8) |
         (static_cast<std::uint32_t>(p[2]) << 16) | (static_cast<std::uint32_t>(p[3]) << 24);
}

float HalfBitsToFloat(std::uint16_t h) {
  const std::uint32_t e = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
  float v;
  if (e == 0) v = std::ldexp(static_cast<float>(mant), -24);
  else if (e == 0x1F) v = mant == 0 ? std::numeric_limits<float>::infinity() : std::numeric_limits<float>::quiet_NaN();
  else v = std::ldexp(1.0F + static_cast<float>(mant) / 1024.0F, static_cast<int>(e) - 15);
  return (h & 0x8000u) ? -v : v;
}

std::size_t ScaleCountOf(const ScaleShape& shape) {
  std::size_t n = 1;
  for (std::size_t d : shape) {
    if (d == 0) throw StageCodecError("scale shape has a zero dimension");
    n = Mul<StageCodecError>(n, d, "scale count");
  }
  return n;
}

// ValidateMatrix of the stage codec (reference stage_codec.cpp:80-137).
void ValidateCodecMatrix(const ProgressiveMatrix& m) {
  const MatrixGeometry& g = m.geometry;
  if (g.original_rows == 0 || g.original_columns == 0) throw StageCodecError("matrix has zero rows or columns");
  if (g.tile_rows == 0 || g.tile_columns == 0 || g.group_size == 0)
    throw StageCodecError("tile shape or group size is zero");
  if (g.tile_columns % g.group_size != 0) throw StageCodecError("group size does not divide the tile width");
  const std::size_t pr = Mul<StageCodecError>(CeilDiv(g.original_rows, g.tile_rows), g.tile_rows, "padded rows");
  const std::size_t pc = Mul<StageCodecError>(CeilDiv(g.original_columns, g.tile_columns), g.tile_columns, "padded columns");
  if (g.padded_rows != pr || g.padded_columns != pc) throw StageCodecError("padded shape is not the shape rounded up to whole tiles");
  if (m.stages.empty() || m.stages.size() > kMaximumStageCount)
    throw StageCodecError("stage count is not in 1..4");
  const ScaleShape shape{g.padded_rows / g.tile_rows, g.padded_columns / g.tile_columns, g.tile_rows,
                         g.tile_columns / g.group_size};
  const std::size_t elements = Mul<StageCodecError>(g.padded_rows, g.padded_columns, "padded element count");
  const std::size_t code_bytes = CeilDiv(elements, 4);
  const std::size_t scale_count = ScaleCountOf(shape);
  for (std::size_t i = 0; i < m.stages.size(); ++i) {
    const DecodedStage& st = m.stages[i];
    if (st.stage_index != i) throw StageCodecError("stage indices are not 0, 1, 2, ... in order");
    if (st.scale_shape != shape || st.scales.size() != scale_count)
      throw StageCodecError("a stage's scale shape differs from the matrix's");
    if (st.packed_codes.size() != code_bytes) throw StageCodecError("a stage's code bytes differ from the matrix's");
    for (float s : st.scales)
      if (!std::isfinite(s) || s < 0.0F) throw StageCodecError("a stage scale is negative, infinite or NaN");
  }
}

std::vector<float> Download(const DeviceArray<float>& d, std::size_t n, cudaStream_t s, const char* what) {
  std::vector<float> out(n);
  if (n != 0) Check(cudaMemcpyAsync(out.data(), d.get(), n * sizeof(float), cudaMemcpyDeviceToHost, s), what);
  Check(cudaStreamSynchronize(s), what);
  return out;
}

// ---- host forms of the reference's host functions ----------------------------------------
//
// DequantizeStage, DequantizePrefix and ProgressiveLinearReference are host functions in
// the reference (stage_codec.cpp:225-339), callable without a GPU.  With a usable device
// they run as raw_dequantize_kernel / raw_linear_ordered_kernel; without one, as the loops
// below, which take the same FP32 operations in the same order (each product and sum
// rounded on its own; this file is compiled with -ffp-contract=off), so both give the
// same bits.  The GEMV entry points have no host form.

bool DeviceUsable() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    static_cast<void>(cudaGetLastError());
    return false;
  }
  return n > 0;
}

int HostCode(const std::vector<std::uint8_t>& codes, std::size_t index) {
  const unsigned raw = (codes[index >> 2] >> (2 * (index & 3))) & 3u;
  return raw >= 2 ? static_cast<int>(raw) - 4 : static_cast<int>(raw);
}

std::size_t HostScaleIndex(const MatrixGeometry& g, std::size_t row, std::size_t col) {
  const std::size_t grid_cols = g.padded_columns / g.tile_columns;
  const std::size_t tr = row / g.tile_rows, rit = row % g.tile_rows;
  const std::size_t tc = col / g.tile_columns, cit = col % g.tile_columns;
  return ((tr * grid_cols + tc) * g.tile_rows + rit) * (g.tile_columns / g.group_size) + cit / g.group_size;
}

// Stages [first, last): the bare product for one stage, else the products added in
// stage order into 0.0f.
std::vector<float> HostDequantize(const ProgressiveMatrix& m, std::size_t first, std::size_t last, bool from_zero) {
  const MatrixGeometry& g = m.geometry;
  std::vector<float> out(g.original_rows * g.original_columns);
  for (std::size_t row = 0; row < g.original_rows; ++row)
    for (std::size_t col = 0; col < g.original_columns; ++col) {
      const std::size_t ci = row * g.padded_columns + col, si = HostScaleIndex(g, row, col);
      float w = 0.0f;
      for (std::size_t s = first; s < last; ++s) {
        const float prod = static_cast<float>(HostCode(m.stages[s].packed_codes, ci)) * m.stages[s].scales[si];
        w = (s == first && !from_zero) ? prod : w + prod;
      }
      out[row * g.original_columns + col] = w;
    }
  return out;
}

// Per (batch, row): per stage a fresh dot summed column by column, added into the
// output; bias last.
std::vector<float> HostLinearOrdered(const ProgressiveMatrix& m, std::size_t prefix, const std::vector<float>& x,
                                     std::size_t batch, const std::vector<float>& bias) {
  const MatrixGeometry& g = m.geometry;
  std::vector<float> y(batch * g.original_rows);
  for (std::size_t b = 0; b < batch; ++b)
    for (std::size_t row = 0; row < g.original_rows; ++row) {
      const float* xb = x.data() + b * g.original_columns;
      float out = 0.0f;
      for (std::size_t s = 0; s < prefix; ++s) {
        float dot = 0.0f;
        for (std::size_t col = 0; col < g.original_columns; ++col) {
          const float w = static_cast<float>(HostCode(m.stages[s].packed_codes, row * g.padded_columns + col)) *
                          m.stages[s].scales[HostScaleIndex(g, row, col)];
          const float p = xb[col] * w;
          dot = dot + p;
        }
        out = out + dot;
      }
      if (!bias.empty()) out = out + bias[row];
      y[b * g.original_rows + row] = out;
    }
  return y;
}

// ---- fused GEMV host validation (reference progressive_gemv.cu:73-183) ------------------

struct HostGeometry {
  std::size_t rows, cols, code_bytes, scale_count;
  ScaleShape shape;
};

HostGeometry ValidateGemvMatrix(const ProgressiveMatrix& m, std::size_t prefix, bool require_fp16) {
  const MatrixGeometry& g = m.geometry;
  if (g.original_rows == 0 || g.original_columns == 0 || g.padded_rows == 0 || g.padded_columns == 0 ||
      g.tile_rows == 0 || g.tile_columns == 0 || g.group_size == 0)
    throw std::invalid_argument("geometry has a zero dimension");
  if (g.tile_columns % g.group_size != 0) throw std::invalid_argument("group size does not divide the tile width");
  const std::size_t pr = Mul<std::overflow_error>(CeilDiv(g.original_rows, g.tile_rows), g.tile_rows, "padded rows");
  const std::size_t pc = Mul<std::overflow_error>(CeilDiv(g.original_columns, g.tile_columns), g.tile_columns, "padded columns");
  if (g.padded_rows != pr || g.padded_columns != pc) throw std::invalid_argument("padded shape is not the shape rounded up to whole tiles");
  if (m.stages.empty() || m.stages.size() > kMaximumStageCount)
    throw std::invalid_argument("stage count is not in 1..4");
  if (prefix > m.stages.size()) throw std::invalid_argument("prefix is deeper than the matrix's stages");
  HostGeometry h{};
  h.rows = g.original_rows;
  h.cols = g.original_columns;
  const std::size_t elements = Mul<std::overflow_error>(g.padded_rows, g.padded_columns, "padded element count");
  Mul<std::overflow_error>(g.original_rows, g.original_columns, "element count");
  h.code_bytes = elements / 4 + (elements % 4 != 0 ? 1U : 0U);
  h.shape = ScaleShape{g.padded_rows / g.tile_rows, g.padded_columns / g.tile_columns, g.tile_rows,
                       g.tile_columns / g.group_size};
  h.scale_count = Mul<std::overflow_error>(h.shape[0], h.shape[1], "scale count over tiles");
  h.scale_count = Mul<std::overflow_error>(h.scale_count, h.shape[2], "scale count over tile rows");
  h.scale_count = Mul<std::overflow_error>(h.scale_count, h.shape[3], "scale count over groups");
  for (std::size_t i = 0; i < m.stages.size(); ++i) {
    const DecodedStage& st = m.stages[i];
    if (st.stage_index != i) throw std::invalid_argument("stage indices are not 0, 1, 2, ... in order");
    if (st.packed_codes.size() != h.code_bytes) throw std::invalid_argument("a stage's code bytes differ from the geometry's");
    if (st.scale_shape != h.shape || st.scales.size() != h.scale_count)
      throw std::invalid_argument("a stage's scale shape differs from the geometry's");
    for (float s : st.scales) {
      if (!std::isfinite(s) || s < 0.0F) throw std::invalid_argument("a stage scale is negative, infinite or NaN");
      if (require_fp16) {
        const float back = __half2float(__float2half_rn(s));
        if (!std::isfinite(back)) throw std::invalid_argument("a stage scale overflows FP16");
        if (back != s) throw std::invalid_argument("a stage scale is not an FP16 value");
      }
    }
  }
  return h;
}

void ValidateFinite(const std::vector<float>& v, const char* what) {
  for (float x : v)
    if (!std::isfinite(x)) throw std::invalid_argument(std::string(what) + " holds an infinite or NaN value");
}

// ---- oracle ------------------------------------------------------------------------------

const char* CublasName(cublasStatus_t s) {
  switch (s) {
    case CUBLAS_STATUS_SUCCESS: return "CUBLAS_STATUS_SUCCESS";
    case CUBLAS_STATUS_NOT_INITIALIZED: return "CUBLAS_STATUS_NOT_INITIALIZED";
    case CUBLAS_STATUS_ALLOC_FAILED: return "CUBLAS_STATUS_ALLOC_FAILED";
    case CUBLAS_STATUS_INVALID_VALUE: return "CUBLAS_STATUS_INVALID_VALUE";
    case CUBLAS_STATUS_ARCH_MISMATCH: return "CUBLAS_STATUS_ARCH_MISMATCH";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "CUBLAS_STATUS_EXECUTION_FAILED";
    case CUBLAS_STATUS_INTERNAL_ERROR: return "CUBLAS_STATUS_INTERNAL_ERROR";
    default: return "CUBLAS_STATUS_OTHER";
  }
}

void CheckBlas(cublasStatus_t s, const char* what) {
  if (s != CUBLAS_STATUS_SUCCESS) throw std::runtime_error(std::string(what) + " failed: " + CublasName(s));
}

class Blas {
 public:
  explicit Blas(cudaStream_t s) {
    CheckBlas(cublasCreate(&h_), "cublasCreate");
    cublasStatus_t st = cublasSetMathMode(h_, CUBLAS_PEDANTIC_MATH);
    if (st == CUBLAS_STATUS_SUCCESS) st = cublasSetAtomicsMode(h_, CUBLAS_ATOMICS_NOT_ALLOWED);
    if (st == CUBLAS_STATUS_SUCCESS) st = cublasSetStream(h_, s);
    if (st != CUBLAS_STATUS_SUCCESS) {
      cublasDestroy(h_);
      h_ = nullptr;
      CheckBlas(st, "configure deterministic cuBLAS");
    }
  }
  ~Blas() {
    if (h_) cublasDestroy(h_);
  }
  Blas(const Blas&) = delete;
  Blas& operator=(const Blas&) = delete;
  cublasHandle_t get() const { return h_; }

 private:
  cublasHandle_t h_ = nullptr;
};

__global__ void AddBias(float* y, const float* bias, std::uint64_t batch, std::uint64_t rows) {
  const std::uint64_t n = batch * rows;
  for (std::uint64_t i = blockIdx.x * static_cast<std::uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<std::uint64_t>(gridDim.x) * blockDim.x)
    y[i] += bias[i % rows];
}

int CublasDim(std::size_t v, const char* what) {
  if (v > static_cast<std::size_t>(std::numeric_limits<int>::max()))
    throw std::invalid_argument(std::string(what) + " is too large for cuBLAS int sizes");
  return static_cast<int>(v);
}

}  // namespace

// ---- stage codec -----------------------------------------------------------------------

DecodedStage DecodeStagePayload(const std::vector<std::uint8_t>& payload, std::uint16_t expected_stage,
                                const ScaleShape& scale_shape) {
  static constexpr std::uint8_t kMagic[8] = {'H', 'Q', 'S', 'T', 'A', 'G', 'E', 0};
  if (payload.size() < 20) throw StageCodecError("payload is shorter than its header");
  if (std::memcmp(payload.data(), kMagic, 8) != 0) throw StageCodecError("payload does not begin with the stage magic");
  const std::uint16_t version = Le16(payload.data() + 8);
  const std::uint16_t stage = Le16(payload.data() + 10);
  const std::size_t code_bytes = Le32(payload.data() + 12);
  const std::size_t scale_count = Le32(payload.data() + 16);
  if (version != kStageCodecVersion) throw StageCodecError("stage codec version not supported: " + std::to_string(version));
  if (stage != expected_stage) throw StageCodecError("payload holds a different stage from the one asked for");
  const std::size_t expected_scales = ScaleCountOf(scale_shape);
  if (scale_count != expected_scales) throw StageCodecError("payload scale count differs from the geometry's");
  const std::size_t scale_bytes = Mul<StageCodecError>(expected_scales, 2, "scale bytes");
  if (code_bytes > std::numeric_limits<std::size_t>::max() - 20 ||
      scale_bytes > std::numeric_limits<std::size_t>::max() - 20 - code_bytes)
    throw StageCodecError("payload size does not fit in size_t");
  if (payload.size() != 20 + code_bytes + scale_bytes) throw StageCodecError("payload size differs from the size its header implies");
  DecodedStage d;
  d.stage_index = stage;
  d.scale_shape = scale_shape;
  d.packed_codes.assign(payload.begin() + 20, payload.begin() + 20 + static_cast<std::ptrdiff_t>(code_bytes));
  d.scales.reserve(expected_scales);
  const std::uint8_t* sp = payload.data() + 20 + code_bytes;
  for (std::size_t i = 0; i < expected_scales; ++i) {
    const float s = HalfBitsToFloat(Le16(sp + 2 * i));
    if (!std::isfinite(s)) throw StageCodecError("a payload scale is infinite or NaN");
    if (s < 0.0F) throw StageCodecError("a payload scale is negative");
    d.scales.push_back(s);
  }
  return d;
}

std::vector<float> DequantizeStage(const ProgressiveMatrix& matrix, std::size_t stage_index) {
  ValidateCodecMatrix(matrix);
  if (stage_index >= matrix.stages.size()) throw StageCodecError("stage index is past the matrix's stages");
  const std::size_t n = Mul<StageCodecError>(matrix.geometry.original_rows, matrix.geometry.original_columns, "output element count");
  if (!DeviceUsable()) return HostDequantize(matrix, stage_index, stage_index + 1, false);
  DeviceArray<float> out(n);
  Stream s;
  DeviceStagesF32 st(matrix, stage_index + 1, s.get());
  const hqb_geometry g = ToGeometry(matrix.geometry);
  Check(hqb_raw_dequantize_stage(&g, st.views.data(), static_cast<std::uint32_t>(matrix.stages.size()),
                                 static_cast<std::uint32_t>(stage_index), out.get(), s.get()),
        "hqb_raw_dequantize_stage");
  return Download(out, n, s.get(), "DequantizeStage");
}

std::vector<float> DequantizePrefix(const ProgressiveMatrix& matrix, std::size_t prefix) {
  ValidateCodecMatrix(matrix);
  if (prefix > matrix.stages.size()) throw StageCodecError("prefix is deeper than the matrix's stages");
  const std::size_t n = Mul<StageCodecError>(matrix.geometry.original_rows, matrix.geometry.original_columns, "output element count");
  if (!DeviceUsable()) return HostDequantize(matrix, 0, prefix, true);
  DeviceArray<float> out(n);
  Stream s;
  DeviceStagesF32 st(matrix, prefix, s.get());
  const hqb_geometry g = ToGeometry(matrix.geometry);
  Check(hqb_raw_dequantize_prefix(&g, st.views.data(), static_cast<std::uint32_t>(matrix.stages.size()),
                                  static_cast<std::uint32_t>(prefix), out.get(), s.get()),
        "hqb_raw_dequantize_prefix");
  return Download(out, n, s.get(), "DequantizePrefix");
}

std::vector<float> ProgressiveLinearReference(const std::vector<float>& inputs, std::size_t batch_size,
                                              const ProgressiveMatrix& matrix, std::size_t prefix,
                                              const std::vector<float>& bias) {
  ValidateCodecMatrix(matrix);
  if (prefix > matrix.stages.size()) throw StageCodecError("prefix is deeper than the matrix's stages");
  const MatrixGeometry& g = matrix.geometry;
  if (inputs.size() != Mul<StageCodecError>(batch_size, g.original_columns, "input element count"))
    throw StageCodecError("input size is not batch x columns");
  if (!bias.empty() && bias.size() != g.original_rows) throw StageCodecError("bias size is not the row count");
  for (float v : inputs)
    if (!std::isfinite(v)) throw StageCodecError("an input or bias value is infinite or NaN");
  for (float v : bias)
    if (!std::isfinite(v)) throw StageCodecError("an input or bias value is infinite or NaN");
  const std::size_t n = Mul<StageCodecError>(batch_size, g.original_rows, "linear output element count");
  if (n == 0) return {};
  if (!DeviceUsable()) return HostLinearOrdered(matrix, prefix, inputs, batch_size, bias);
  Stream s;
  DeviceArray<float> x(inputs.size()), b(bias.size()), y(n);
  Upload(x, inputs, s.get(), "cudaMemcpyAsync(inputs H2D)");
  Upload(b, bias, s.get(), "cudaMemcpyAsync(bias H2D)");
  DeviceStagesF32 st(matrix, prefix, s.get());
  const hqb_geometry hg = ToGeometry(g);
  Check(hqb_raw_linear_ordered(&hg, st.views.data(), static_cast<std::uint32_t>(matrix.stages.size()),
                               static_cast<std::uint32_t>(prefix), x.get(), batch_size,
                               bias.empty() ? nullptr : b.get(), y.get(), s.get()),
        "hqb_raw_linear_ordered");
  return Download(y, n, s.get(), "ProgressiveLinearReference");
}

std::uint32_t Crc32c(const std::uint8_t* data, std::size_t size, std::uint32_t crc) {
  if (data == nullptr && size != 0) throw std::invalid_argument("CRC32C given a null pointer with a non-zero size");
  static const auto table = [] {
    std::array<std::uint32_t, 256> t{};
    for (std::uint32_t i = 0; i < 256; ++i) {
      std::uint32_t v = i;
      for (int k = 0; k < 8; ++k) v = (v >> 1) ^ ((v & 1U) ? 0x82F63B78U : 0U);
      t[i] = v;
    }
    return t;
  }();
  std::uint32_t v = crc ^ 0xFFFFFFFFU;
  for (std::size_t i = 0; i < size; ++i) v = table[(v ^ data[i]) & 0xFFU] ^ (v >> 8);
  return v ^ 0xFFFFFFFFU;
}

// ---- fused GEMV --------------------------------------------------------------------------

cudaError_t LaunchProgressiveGemv(const ProgressiveGemvIoDeviceView& io, const ProgressiveGemvDeviceView& matrix,
                                  std::size_t prefix, cudaStream_t stream) noexcept {
  if (matrix.stage_count == 0 || matrix.stage_count > kMaximumStageCount || prefix > matrix.stage_count)
    return cudaErrorInvalidValue;
  hqb_geometry g;
  std::memcpy(&g, &matrix.geometry, sizeof(g));
  hqb_raw_stage st[kMaximumStageCount];
  std::memcpy(st, matrix.stages, sizeof(st));
  return static_cast<cudaError_t>(hqb_raw_gemv(&g, st, static_cast<std::uint32_t>(matrix.stage_count),
                                               static_cast<std::uint32_t>(prefix), io.input, io.input_count, io.bias,
                                               io.bias_count, io.output, io.output_count, stream));
}

std::vector<float> ProgressiveGemvCuda(const std::vector<float>& input, const ProgressiveMatrix& matrix,
                                       std::size_t prefix, const std::vector<float>& bias) {
  const HostGeometry h = ValidateGemvMatrix(matrix, prefix, true);
  if (input.size() != h.cols) throw std::invalid_argument("input size is not the column count");
  if (!bias.empty() && bias.size() != h.rows) throw std::invalid_argument("bias size is not the row count");
  ValidateFinite(input, "input");
  ValidateFinite(bias, "bias");
  DeviceArray<float> x(input.size()), y(h.rows), b(bias.size());
  std::vector<DeviceArray<std::uint8_t>> codes(kMaximumStageCount);
  std::vector<DeviceArray<std::uint16_t>> scales(kMaximumStageCount);
  std::vector<std::vector<std::uint16_t>> bits(kMaximumStageCount);
  Stream s;  // declared after the buffers: drains queued work first on every exit
  Upload(x, input, s.get(), "cudaMemcpyAsync(input H2D)");
  Upload(b, bias, s.get(), "cudaMemcpyAsync(bias H2D)");
  ProgressiveGemvDeviceView view{};
  view.geometry = {h.rows, h.cols, matrix.geometry.padded_rows, matrix.geometry.padded_columns,
                   matrix.geometry.tile_rows, matrix.geometry.tile_columns, matrix.geometry.group_size};
  view.stage_count = matrix.stages.size();
  for (std::size_t i = 0; i < prefix; ++i) {
    const DecodedStage& st = matrix.stages[i];
    bits[i].reserve(st.scales.size());
    for (float v : st.scales) bits[i].push_back(static_cast<__half_raw>(__float2half_rn(v)).x);
    codes[i] = DeviceArray<std::uint8_t>(st.packed_codes.size());
    scales[i] = DeviceArray<std::uint16_t>(bits[i].size());
    Upload(codes[i], st.packed_codes, s.get(), "cudaMemcpyAsync(stage codes H2D)");
    Upload(scales[i], bits[i], s.get(), "cudaMemcpyAsync(stage scales H2D)");
    view.stages[i] = {codes[i].get(), st.packed_codes.size(), scales[i].get(), bits[i].size()};
  }
  const ProgressiveGemvIoDeviceView io{x.get(), input.size(), bias.empty() ? nullptr : b.get(), bias.size(), y.get(), h.rows};
  Check(LaunchProgressiveGemv(io, view, prefix, s.get()), "progressive GEMV launch");
  return Download(y, h.rows, s.get(), "progressive GEMV execution");
}

// ---- CUDA oracle -------------------------------------------------------------------------

bool CudaDeviceAvailable(std::string* reason) noexcept {
  try {
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      if (reason) *reason = std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
      static_cast<void>(cudaGetLastError());
      return false;
    }
    if (n <= 0) {
      if (reason) *reason = "CUDA runtime reported no devices";
      return false;
    }
    if (reason) reason->clear();
    return true;
  } catch (...) {
    return false;
  }
}

std::vector<float> ProgressiveLinearCudaOracle(const std::vector<float>& inputs, std::size_t batch_size,
                                               const ProgressiveMatrix& matrix, std::size_t prefix,
                                               const std::vector<float>& bias) {
  const HostGeometry h = ValidateGemvMatrix(matrix, prefix, false);
  if (inputs.size() != Mul<std::overflow_error>(batch_size, h.cols, "input"))
    throw std::invalid_argument("input size is not batch x columns");
  if (!bias.empty() && bias.size() != h.rows) throw std::invalid_argument("bias size is not the row count");
  ValidateFinite(inputs, "inputs");
  ValidateFinite(bias, "bias");
  if (batch_size == 0) return {};
  const std::size_t n_out = Mul<std::overflow_error>(batch_size, h.rows, "output");
  const int rows = CublasDim(h.rows, "output feature count");
  const int cols = CublasDim(h.cols, "input feature count");
  const int batch = CublasDim(batch_size, "batch size");
  DeviceArray<float> w(h.rows * h.cols), x(inputs.size()), y(n_out), b(bias.size());
  Stream s;
  Upload(x, inputs, s.get(), "cudaMemcpyAsync(inputs H2D)");
  Upload(b, bias, s.get(), "cudaMemcpyAsync(bias H2D)");
  DeviceStagesF32 st(matrix, prefix, s.get());
  const hqb_geometry g = ToGeometry(matrix.geometry);
  Check(hqb_raw_dequantize_prefix(&g, st.views.data(), static_cast<std::uint32_t>(matrix.stages.size()),
                                  static_cast<std::uint32_t>(prefix), w.get(), s.get()),
        "hqb_raw_dequantize_prefix");
  Blas blas(s.get());
  const float one = 1.0F, zero = 0.0F;
  // Row-major W[O,I] is column-major [I,O]; Y_col[O,B] = Wᵀ X has the storage of row-major Y[B,O].
  CheckBlas(cublasSgemm(blas.get(), CUBLAS_OP_T, CUBLAS_OP_N, rows, batch, cols, &one, w.get(), cols, x.get(), cols,
                        &zero, y.get(), rows),
            "cublasSgemm(progressive linear oracle)");
  if (!bias.empty()) {
    AddBias<<<static_cast<unsigned>(std::min<std::size_t>((n_out + 255) / 256, 65535)), 256, 0, s.get()>>>(
        y.get(), b.get(), batch_size, h.rows);
    Check(cudaGetLastError(), "AddBias launch");
  }
  return Download(y, n_out, s.get(), "ProgressiveLinearCudaOracle");
}

}  // namespace harpq::native_runtime
