// C++ API contract test, linked against libharpq_b200.so (built by harp-q_b200/build.py,
// run by tests/test_gpu_native.py).  Covers the reference's native surface
// (harpq::native_runtime) and the plane-layout C ABI called from C++.
// Exit 0 on success, 77 when no CUDA device is present, 1 on failure.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

#include "harpq/cuda_oracle.hpp"
#include "harpq/native/stage_codec.hpp"
#include "harpq/progressive_gemv.hpp"
#include "harpq_b200.h"

namespace nr = harpq::native_runtime;

namespace {

int failures = 0;

void Expect(bool ok, const std::string& what) {
  if (!ok) {
    std::fprintf(stderr, "FAIL: %s\n", what.c_str());
    ++failures;
  }
}

template <typename E>
void ExpectThrows(const std::function<void()>& f, const std::string& what) {
  try {
    f();
  } catch (const E&) {
    return;
  } catch (const std::exception& e) {
    Expect(false, what + " threw the wrong exception: " + e.what());
    return;
  }
  Expect(false, what + " did not throw");
}

std::uint32_t Hash(std::uint64_t v) {
  v ^= v >> 33;
  v *= 0xff51afd7ed558ccdULL;
  v ^= v >> 33;
  v *= 0xc4ceb9fe1a85ec53ULL;
  v ^= v >> 33;
  return static_cast<std::uint32_t>(v);
}

// Deterministic matrix with FP16-exact scales.
nr::ProgressiveMatrix MakeMatrix(std::size_t rows, std::size_t cols, std::size_t tr, std::size_t tc, std::size_t grp,
                                 std::size_t stages) {
  nr::ProgressiveMatrix m{};
  const std::size_t pr = (rows + tr - 1) / tr * tr, pc = (cols + tc - 1) / tc * tc;
  m.geometry = {rows, cols, pr, pc, tr, tc, grp};
  const nr::ScaleShape shape{pr / tr, pc / tc, tr, tc / grp};
  const std::size_t nscale = shape[0] * shape[1] * shape[2] * shape[3];
  for (std::size_t s = 0; s < stages; ++s) {
    nr::DecodedStage st{};
    st.stage_index = static_cast<std::uint16_t>(s);
    st.scale_shape = shape;
    st.packed_codes.resize((pr * pc + 3) / 4);
    for (std::size_t i = 0; i < st.packed_codes.size(); ++i) st.packed_codes[i] = static_cast<std::uint8_t>(Hash(i * 7 + s));
    for (std::size_t i = 0; i < nscale; ++i)
      st.scales.push_back(std::ldexp(static_cast<float>(1 + Hash(i + 1000 * s) % 1024) / 1024.0F + 1.0F,
                                     -6 - static_cast<int>(s) - static_cast<int>(Hash(i) % 3)));
    m.stages.push_back(std::move(st));
  }
  return m;
}

std::vector<std::uint8_t> EncodePayload(const nr::DecodedStage& st) {
  std::vector<std::uint8_t> p = {'H', 'Q', 'S', 'T', 'A', 'G', 'E', 0, 1, 0};
  const auto put16 = [&](std::uint32_t v) {
    p.push_back(v & 0xFF);
    p.push_back((v >> 8) & 0xFF);
  };
  const auto put32 = [&](std::uint32_t v) {
    put16(v & 0xFFFF);
    put16(v >> 16);
  };
  p.resize(10);
  put16(st.stage_index);
  put32(static_cast<std::uint32_t>(st.packed_codes.size()));
  put32(static_cast<std::uint32_t>(st.scales.size()));
  p.insert(p.end(), st.packed_codes.begin(), st.packed_codes.end());
  for (float s : st.scales) put16(static_cast<__half_raw>(__float2half_rn(s)).x);
  return p;
}

int Code(const nr::DecodedStage& st, std::size_t i) {
  const int raw = (st.packed_codes[i / 4] >> (2 * (i % 4))) & 3;
  return raw >= 2 ? raw - 4 : raw;
}

float ScaleAt(const nr::ProgressiveMatrix& m, const nr::DecodedStage& st, std::size_t r, std::size_t c) {
  const auto& g = m.geometry;
  const std::size_t gc = g.padded_columns / g.tile_columns, groups = g.tile_columns / g.group_size;
  return st.scales[((r / g.tile_rows * gc + c / g.tile_columns) * g.tile_rows + r % g.tile_rows) * groups +
                   (c % g.tile_columns) / g.group_size];
}

// Host restatement used only as this test's expectation.
std::vector<float> HostPrefix(const nr::ProgressiveMatrix& m, std::size_t prefix) {
  const auto& g = m.geometry;
  std::vector<float> w(g.original_rows * g.original_columns, 0.0F);
  for (std::size_t s = 0; s < prefix; ++s)
    for (std::size_t r = 0; r < g.original_rows; ++r)
      for (std::size_t c = 0; c < g.original_columns; ++c)
        w[r * g.original_columns + c] +=
            static_cast<float>(Code(m.stages[s], r * g.padded_columns + c)) * ScaleAt(m, m.stages[s], r, c);
  return w;
}

bool Near(const std::vector<float>& a, const std::vector<float>& e, float atol, float rtol) {
  if (a.size() != e.size()) return false;
  for (std::size_t i = 0; i < a.size(); ++i)
    if (!std::isfinite(a[i]) || std::fabs(a[i] - e[i]) > atol + rtol * std::fabs(e[i])) return false;
  return true;
}

void TestCrcAndPayload() {
  const char* digits = "123456789";
  const auto* b = reinterpret_cast<const std::uint8_t*>(digits);
  Expect(nr::Crc32c(b, 9) == 0xE3069283U, "CRC32C standard vector");
  Expect(nr::Crc32c(b + 4, 5, nr::Crc32c(b, 4)) == 0xE3069283U, "CRC32C incremental");
  Expect(nr::Crc32c(nullptr, 0) == 0U, "CRC32C empty");
  ExpectThrows<std::invalid_argument>([] { (void)nr::Crc32c(nullptr, 1); }, "CRC32C null data");

  const nr::ProgressiveMatrix m = MakeMatrix(37, 70, 16, 32, 8, 2);
  for (std::size_t s = 0; s < 2; ++s) {
    const auto payload = EncodePayload(m.stages[s]);
    const nr::DecodedStage d = nr::DecodeStagePayload(payload, static_cast<std::uint16_t>(s), m.stages[s].scale_shape);
    Expect(d.packed_codes == m.stages[s].packed_codes && d.scales == m.stages[s].scales, "payload round trip");
    auto bad = payload;
    bad[8] = 2;
    ExpectThrows<nr::StageCodecError>([&] { (void)nr::DecodeStagePayload(bad, 0, m.stages[s].scale_shape); }, "bad version");
    ExpectThrows<nr::StageCodecError>(
        [&] { (void)nr::DecodeStagePayload(payload, static_cast<std::uint16_t>(s + 1), m.stages[s].scale_shape); },
        "stage mismatch");
    bad = payload;
    bad.pop_back();
    ExpectThrows<nr::StageCodecError>([&] { (void)nr::DecodeStagePayload(bad, static_cast<std::uint16_t>(s), m.stages[s].scale_shape); },
                                      "short payload");
  }
}

void TestDecodeAndReferenceExact() {
  for (const auto& m : {MakeMatrix(37, 70, 16, 32, 8, 4), MakeMatrix(200, 300, 128, 128, 128, 4)}) {
    for (std::size_t p = 0; p <= 4; ++p) {
      const auto w = nr::DequantizePrefix(m, p);
      const auto host = HostPrefix(m, p);
      Expect(w.size() == host.size() && std::memcmp(w.data(), host.data(), w.size() * 4) == 0, "DequantizePrefix bit-exact");
    }
    const auto& g = m.geometry;
    std::vector<float> x(2 * g.original_columns);
    for (std::size_t i = 0; i < x.size(); ++i) x[i] = static_cast<float>(static_cast<int>(Hash(i) % 200) - 100) / 37.0F;
    std::vector<float> bias(g.original_rows, 0.25F);
    const auto y = nr::ProgressiveLinearReference(x, 2, m, 3, bias);
    // scalar order: stage-major fresh dots, bias last
    std::vector<float> e(2 * g.original_rows, 0.0F);
    for (std::size_t s = 0; s < 3; ++s) {
      const auto ws = nr::DequantizeStage(m, s);
      for (std::size_t b = 0; b < 2; ++b)
        for (std::size_t r = 0; r < g.original_rows; ++r) {
          float dot = 0.0F;
          for (std::size_t c = 0; c < g.original_columns; ++c) {
            const float prod = x[b * g.original_columns + c] * ws[r * g.original_columns + c];
            dot = dot + prod;
          }
          e[b * g.original_rows + r] += dot;
        }
    }
    for (std::size_t b = 0; b < 2; ++b)
      for (std::size_t r = 0; r < g.original_rows; ++r) e[b * g.original_rows + r] += bias[r];
    Expect(std::memcmp(y.data(), e.data(), y.size() * 4) == 0, "ProgressiveLinearReference bit-exact");
  }
}

void TestFusedAgainstOracle() {
  for (const auto& m : {MakeMatrix(37, 70, 16, 32, 8, 4), MakeMatrix(200, 300, 128, 128, 128, 4),
                        MakeMatrix(3, 513, 4, 128, 128, 4)}) {
    const auto& g = m.geometry;
    std::vector<float> x(g.original_columns), bias(g.original_rows);
    for (std::size_t i = 0; i < x.size(); ++i) x[i] = static_cast<float>(static_cast<int>(Hash(i + 9) % 101) - 50) / 25.0F;
    for (std::size_t i = 0; i < bias.size(); ++i) bias[i] = static_cast<float>(i % 5) / 8.0F;
    for (std::size_t p = 0; p <= 4; ++p) {
      const auto fused = nr::ProgressiveGemvCuda(x, m, p, bias);
      const auto oracle = nr::ProgressiveLinearCudaOracle(x, 1, m, p, bias);
      Expect(Near(fused, oracle, 2e-4F, 2e-4F), "fused GEMV vs cuBLAS oracle prefix " + std::to_string(p));
    }
  }
  const nr::ProgressiveMatrix m = MakeMatrix(37, 70, 16, 32, 8, 4);
  const std::vector<float> x(70, 0.5F);
  Expect(nr::ProgressiveLinearCudaOracle({}, 0, m, 4).empty(), "oracle empty batch");
  ExpectThrows<std::invalid_argument>([&] { (void)nr::ProgressiveGemvCuda(x, m, 5); }, "prefix range");
  ExpectThrows<std::invalid_argument>([&] { (void)nr::ProgressiveGemvCuda({}, m, 1); }, "input size");
  auto inexact = m;
  inexact.stages[0].scales[0] = 0.1F;
  ExpectThrows<std::invalid_argument>([&] { (void)nr::ProgressiveGemvCuda(x, inexact, 1); }, "inexact FP16 scale");
  auto overflow = m;
  overflow.geometry = {std::numeric_limits<std::size_t>::max(), std::numeric_limits<std::size_t>::max(),
                       std::numeric_limits<std::size_t>::max(), std::numeric_limits<std::size_t>::max(), 1, 1, 1};
  ExpectThrows<std::overflow_error>([&] { (void)nr::ProgressiveGemvCuda(x, overflow, 1); }, "overflowing geometry");
}

void TestPlaneAbiFromCpp() {
  const nr::ProgressiveMatrix m = MakeMatrix(260, 390, 128, 128, 128, 4);
  const auto& gm = m.geometry;
  hqb_geometry g{gm.original_rows, gm.original_columns, gm.padded_rows, gm.padded_columns, 128, 128, 128};
  const std::uint64_t pb = hqb_plane_bytes(&g);
  Expect(pb == 3 * 4 * 4352ULL, "plane bytes");
  hqb_plane_matrix pm{gm.original_rows, gm.original_columns, 3, 4, 4, 0, {}};
  std::vector<void*> owned;
  for (std::size_t s = 0; s < 4; ++s) {
    void *codes = nullptr, *bits = nullptr, *plane = nullptr;
    cudaMalloc(&codes, m.stages[s].packed_codes.size());
    cudaMalloc(&bits, m.stages[s].scales.size() * 2);
    cudaMalloc(&plane, pb);
    std::vector<std::uint16_t> hb;
    for (float v : m.stages[s].scales) hb.push_back(static_cast<__half_raw>(__float2half_rn(v)).x);
    cudaMemcpy(codes, m.stages[s].packed_codes.data(), m.stages[s].packed_codes.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(bits, hb.data(), hb.size() * 2, cudaMemcpyHostToDevice);
    const hqb_raw_stage st{static_cast<const std::uint8_t*>(codes), m.stages[s].packed_codes.size(),
                           static_cast<const std::uint16_t*>(bits), hb.size()};
    Expect(hqb_repack_stage(&g, &st, plane, nullptr, nullptr) == 0, "repack");
    pm.planes[s] = plane;
    owned.insert(owned.end(), {codes, bits, plane});
  }
  std::vector<float> x(390);
  for (std::size_t i = 0; i < x.size(); ++i) x[i] = static_cast<float>(static_cast<int>(Hash(i) % 61) - 30) / 16.0F;
  const std::uint64_t wsb = hqb_workspace_bytes(&pm, 1, HQB_F32, 0);
  void *ws = nullptr, *dx = nullptr, *dy = nullptr;
  cudaMalloc(&ws, wsb);
  cudaMalloc(&dx, x.size() * 4);
  cudaMalloc(&dy, 260 * 4);
  cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice);
  Expect(hqb_workspace_init(ws, wsb, nullptr) == 0, "workspace init");
  for (std::uint32_t p = 1; p <= 4; ++p) {
    Expect(hqb_gemv(&pm, p, dx, HQB_F32, 1, nullptr, HQB_F32, dy, HQB_F32, ws, wsb, nullptr) == 0, "hqb_gemv");
    std::vector<float> y(260);
    cudaMemcpy(y.data(), dy, 260 * 4, cudaMemcpyDeviceToHost);
    const auto e = nr::ProgressiveLinearCudaOracle(x, 1, m, p);
    Expect(Near(y, e, 2e-4F, 2e-4F), "plane GEMV vs oracle prefix " + std::to_string(p));
  }
  int flags = -1;
  Expect(hqb_workspace_error(ws, &flags, nullptr) == 0 && flags == 0, "workspace error word");
  Expect(hqb_gemv(&pm, 5, dx, HQB_F32, 1, nullptr, HQB_F32, dy, HQB_F32, ws, wsb, nullptr) == HQB_ERR_INVALID,
         "prefix > stage_count rejected");
  for (void* p : owned) cudaFree(p);
  cudaFree(ws);
  cudaFree(dx);
  cudaFree(dy);
}

}  // namespace

int main() {
  std::string why;
  if (!nr::CudaDeviceAvailable(&why)) {
    std::printf("SKIP: no CUDA device: %s\n", why.c_str());
    return 77;
  }
  try {
    TestCrcAndPayload();
    TestDecodeAndReferenceExact();
    TestFusedAgainstOracle();
    TestPlaneAbiFromCpp();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "FAIL: unexpected exception: %s\n", e.what());
    return 1;
  }
  if (failures != 0) {
    std::fprintf(stderr, "%d check(s) failed\n", failures);
    return 1;
  }
  std::printf("hqb C++ API tests passed\n");
  return 0;
}
