// TEST INFRASTRUCTURE ONLY — C shim over the reference's own C++ stage codec.
//
// oracle/build.py compiles this file together with the reference's unmodified
// native/src/stage_codec.cpp (read from the reference checkout, never copied into
// this repository) into oracle/_ref/libharpq_ref.so.  Tests use it to pin the C
// restatement in harpq_oracle.c; bench.py's reference arm times
// ProgressiveLinearReference through it.  Everything except the hqr_* functions
// is compiled with hidden visibility so its harpq::native_runtime symbols can
// never interpose on the product library's.
#include "harpq/native/stage_codec.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <new>
#include <vector>

namespace nr = harpq::native_runtime;

#define HQR_API extern "C" __attribute__((visibility("default")))

struct hqr_geometry {
  std::uint64_t v[7];
};

struct hqr_stage {
  const std::uint8_t* codes;
  std::uint64_t code_bytes;
  const float* scales;
  std::uint64_t scale_count;
};

namespace {
nr::ProgressiveMatrix Build(const hqr_geometry* g, const hqr_stage* s, std::uint32_t n) {
  nr::ProgressiveMatrix m{};
  m.geometry = {g->v[0], g->v[1], g->v[2], g->v[3], g->v[4], g->v[5], g->v[6]};
  const nr::ScaleShape shape{g->v[2] / g->v[4], g->v[3] / g->v[5], g->v[4], g->v[5] / g->v[6]};
  for (std::uint32_t i = 0; i < n; ++i) {
    nr::DecodedStage st;
    st.stage_index = static_cast<std::uint16_t>(i);
    st.packed_codes.assign(s[i].codes, s[i].codes + s[i].code_bytes);
    st.scales.assign(s[i].scales, s[i].scales + s[i].scale_count);
    st.scale_shape = shape;
    m.stages.push_back(std::move(st));
  }
  return m;
}
}  // namespace

HQR_API std::uint32_t hqr_crc32c(const std::uint8_t* data, std::uint64_t size, std::uint32_t crc) {
  return nr::Crc32c(data, size, crc);
}

// Returns 0 on success, 1 when DecodeStagePayload throws StageCodecError.
HQR_API int hqr_decode_payload(const std::uint8_t* payload, std::uint64_t size,
                               std::uint16_t stage, const std::uint64_t* scale_shape,
                               std::uint8_t* codes_out, float* scales_out) {
  try {
    const std::vector<std::uint8_t> bytes(payload, payload + size);
    const nr::ScaleShape shape{scale_shape[0], scale_shape[1], scale_shape[2], scale_shape[3]};
    const nr::DecodedStage d = nr::DecodeStagePayload(bytes, stage, shape);
    std::memcpy(codes_out, d.packed_codes.data(), d.packed_codes.size());
    std::memcpy(scales_out, d.scales.data(), d.scales.size() * sizeof(float));
    return 0;
  } catch (const nr::StageCodecError&) {
    return 1;
  } catch (...) {
    return 2;
  }
}

// An owned ProgressiveMatrix, built once so a timed loop measures only the
// reference arithmetic.
HQR_API void* hqr_matrix_create(const hqr_geometry* g, const hqr_stage* s, std::uint32_t n) {
  try {
    return new nr::ProgressiveMatrix(Build(g, s, n));
  } catch (...) {
    return nullptr;
  }
}

HQR_API void hqr_matrix_free(void* m) { delete static_cast<nr::ProgressiveMatrix*>(m); }

HQR_API int hqr_dequantize_prefix(void* m, std::uint32_t prefix, float* out) {
  try {
    const std::vector<float> w = nr::DequantizePrefix(*static_cast<nr::ProgressiveMatrix*>(m), prefix);
    std::memcpy(out, w.data(), w.size() * sizeof(float));
    return 0;
  } catch (const nr::StageCodecError&) {
    return 1;
  } catch (...) {
    return 2;
  }
}

HQR_API int hqr_linear_reference(void* m, std::uint32_t prefix, const float* inputs,
                                 std::uint64_t batch, const float* bias, float* out) {
  try {
    const auto& mat = *static_cast<nr::ProgressiveMatrix*>(m);
    const std::vector<float> x(inputs, inputs + batch * mat.geometry.original_columns);
    std::vector<float> b;
    if (bias != nullptr) b.assign(bias, bias + mat.geometry.original_rows);
    const std::vector<float> y = nr::ProgressiveLinearReference(x, batch, mat, prefix, b);
    std::memcpy(out, y.data(), y.size() * sizeof(float));
    return 0;
  } catch (const nr::StageCodecError&) {
    return 1;
  } catch (...) {
    return 2;
  }
}
