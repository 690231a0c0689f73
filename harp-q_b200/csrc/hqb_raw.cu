// Kernels on the reference's own device layout (any tile geometry): the drop-in
// batch-one GEMV behind LaunchProgressiveGemv, exact-order stage/prefix decode and
// the reference's scalar-order linear.
//
// Layout (reference native/src/progressive_gemv.cu:359-392): codes row-major over the
// padded matrix, element (r, c) at byte (r*padded_cols + c)/4, bits 2*((r*padded_cols + c)%4);
// scale of (r, c) at [r/tile_rows][c/tile_cols][r%tile_rows][(c%tile_cols)/group].
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "harpq_b200.h"
#include "hqb_internal.h"

namespace hqb {
namespace {

struct RawGeo {
  uint64_t rows, cols, padded_rows, padded_cols;
  uint32_t tile_rows, tile_cols, group, grid_cols, groups_per_tile;
};

struct RawStages {
  const uint8_t* codes[HQB_MAX_STAGES];
  const void* scales[HQB_MAX_STAGES];  // FP16 bits or FP32, by kernel
};

__device__ __forceinline__ int code_at(const uint8_t* codes, uint64_t index) {
  const uint32_t raw = (codes[index >> 2] >> (2 * (index & 3))) & 3u;
  return raw >= 2 ? static_cast<int>(raw) - 4 : static_cast<int>(raw);
}

__device__ __forceinline__ uint64_t scale_index(const RawGeo& g, uint64_t row, uint64_t col) {
  const uint64_t tr = row / g.tile_rows, rit = row - tr * g.tile_rows;
  const uint64_t tc = col / g.tile_cols, cit = col - tc * g.tile_cols;
  return ((tr * g.grid_cols + tc) * g.tile_rows + rit) * g.groups_per_tile + cit / g.group;
}

__device__ __forceinline__ float scale_of(const void* s, uint64_t i, bool fp16) {
  return fp16 ? __half2float(__ushort_as_half(static_cast<const uint16_t*>(s)[i])) : static_cast<const float*>(s)[i];
}

// One warp per output row.  When group % 4 == 0 every byte (4 codes) shares one scale
// per stage and a lane consumes one byte per stage and step (128 columns per warp
// step, one 32-byte sector per stage); otherwise the lane walks single columns.
// Weight of a column: fmaf(code, scale, w) over the stages in order; then
// fmaf(x, w, sum) — the reference's per-element arithmetic (progressive_gemv.cu:375-392).
template <bool kByteGroups>
__global__ void __launch_bounds__(256) raw_gemv_kernel(RawGeo g, RawStages st, uint32_t prefix,
                                                       const float* __restrict__ x,
                                                       const float* __restrict__ bias,
                                                       float* __restrict__ y) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x >> 5);
  for (uint64_t row = blockIdx.x * static_cast<uint64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); row < g.rows;
       row += warps) {
    float sum = 0.0f;
    const uint64_t base = row * g.padded_cols;
    if constexpr (kByteGroups) {
      for (uint64_t col0 = 4ull * lane; col0 < g.cols; col0 += 128) {
        uint32_t bytes[HQB_MAX_STAGES];
        float sc[HQB_MAX_STAGES];
        const uint64_t si = scale_index(g, row, col0);
#pragma unroll
        for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) {
          if (s < prefix) {
            bytes[s] = st.codes[s][(base + col0) >> 2];
            sc[s] = scale_of(st.scales[s], si, true);
          }
        }
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
          if (col0 + k >= g.cols) break;
          float w = 0.0f;
#pragma unroll
          for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) {
            if (s < prefix) {
              const uint32_t raw = (bytes[s] >> (2 * k)) & 3u;
              const int code = raw >= 2 ? static_cast<int>(raw) - 4 : static_cast<int>(raw);
              w = fmaf(static_cast<float>(code), sc[s], w);
            }
          }
          sum = fmaf(x[col0 + k], w, sum);
        }
      }
    } else {
      for (uint64_t col = lane; col < g.cols; col += 32) {
        const uint64_t si = scale_index(g, row, col);
        float w = 0.0f;
#pragma unroll
        for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s)
          if (s < prefix) w = fmaf(static_cast<float>(code_at(st.codes[s], base + col)), scale_of(st.scales[s], si, true), w);
        sum = fmaf(x[col], w, sum);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) y[row] = sum + (bias == nullptr ? 0.0f : bias[row]);
  }
}

// DequantizeStage (from_zero == false: the bare product) or DequantizePrefix
// (from_zero == true: products added in stage order into 0.0f).
__global__ void raw_dequantize_kernel(RawGeo g, RawStages st, uint32_t first, uint32_t last, int from_zero,
                                      float* __restrict__ out) {
  const uint64_t n = g.rows * g.cols;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t row = i / g.cols, col = i - row * g.cols;
    const uint64_t ci = row * g.padded_cols + col;
    const uint64_t si = scale_index(g, row, col);
    float w = 0.0f;
    for (uint32_t s = first; s < last; ++s) {
      const float prod = __fmul_rn(static_cast<float>(code_at(st.codes[s], ci)), scale_of(st.scales[s], si, false));
      w = (s == first && !from_zero) ? prod : __fadd_rn(w, prod);
    }
    out[i] = w;
  }
}

// ProgressiveLinearReference order: one thread per (batch, row); per stage a fresh dot
// summed column by column, added into the output; bias last.  Every operation is a
// separately rounded FP32 multiply or add (no contraction), as on the reference's CPU.
__global__ void raw_linear_ordered_kernel(RawGeo g, RawStages st, uint32_t prefix, const float* __restrict__ x,
                                          uint64_t batch, const float* __restrict__ bias, float* __restrict__ y) {
  const uint64_t n = batch * g.rows;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t b = i / g.rows, row = i - b * g.rows;
    const float* xb = x + b * g.cols;
    float out = 0.0f;
    for (uint32_t s = 0; s < prefix; ++s) {
      float dot = 0.0f;
      for (uint64_t col = 0; col < g.cols; ++col) {
        const float w = __fmul_rn(static_cast<float>(code_at(st.codes[s], row * g.padded_cols + col)),
                                  scale_of(st.scales[s], scale_index(g, row, col), false));
        dot = __fadd_rn(dot, __fmul_rn(xb[col], w));
      }
      out = __fadd_rn(out, dot);
    }
    if (bias != nullptr) out = __fadd_rn(out, bias[row]);
    y[i] = out;
  }
}

// Scalar validation of LaunchProgressiveGemv's device view (reference
// native/src/progressive_gemv.cu:266-321): the same fields, the same overflow checks.
bool geometry_ok(const hqb_geometry* gm, uint64_t* code_bytes, uint64_t* scale_count) {
  if (gm->original_rows == 0 || gm->original_columns == 0 || gm->padded_rows == 0 || gm->padded_columns == 0 ||
      gm->tile_rows == 0 || gm->tile_columns == 0 || gm->group_size == 0 || gm->tile_columns % gm->group_size != 0)
    return false;
  const uint64_t grid_rows = gm->original_rows / gm->tile_rows + (gm->original_rows % gm->tile_rows != 0);
  const uint64_t grid_cols = gm->original_columns / gm->tile_columns + (gm->original_columns % gm->tile_columns != 0);
  uint64_t pr = 0, pc = 0, pe = 0, sg = 0;
  if (!mul_ok(grid_rows, gm->tile_rows, &pr) || !mul_ok(grid_cols, gm->tile_columns, &pc) || pr != gm->padded_rows ||
      pc != gm->padded_columns || !mul_ok(gm->padded_rows, gm->padded_columns, &pe) || !mul_ok(grid_rows, grid_cols, &sg) ||
      !mul_ok(sg, gm->tile_rows, &sg) || !mul_ok(sg, gm->tile_columns / gm->group_size, &sg))
    return false;
  *code_bytes = pe / 4 + (pe % 4 != 0);
  *scale_count = sg;
  return true;
}

bool to_raw_geo(const hqb_geometry* gm, RawGeo* out) {
  // kernels index tiles with 32-bit tile geometry
  if (gm->tile_rows > 0xFFFFFFFFull || gm->tile_columns > 0xFFFFFFFFull) return false;
  out->rows = gm->original_rows;
  out->cols = gm->original_columns;
  out->padded_rows = gm->padded_rows;
  out->padded_cols = gm->padded_columns;
  out->tile_rows = static_cast<uint32_t>(gm->tile_rows);
  out->tile_cols = static_cast<uint32_t>(gm->tile_columns);
  out->group = static_cast<uint32_t>(gm->group_size);
  out->grid_cols = static_cast<uint32_t>(gm->padded_columns / gm->tile_columns);
  out->groups_per_tile = static_cast<uint32_t>(gm->tile_columns / gm->group_size);
  return true;
}

unsigned grid_for(uint64_t n, unsigned per_block) {
  return static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>((n + per_block - 1) / per_block, 65535ull * 8)));
}

int f32_stages(const hqb_geometry* gm, const hqb_raw_stage_f32* stages, uint32_t stage_count, uint32_t needed,
               RawGeo* g, RawStages* st) {
  uint64_t cb = 0, sc = 0;
  if (gm == nullptr || stages == nullptr || stage_count == 0 || stage_count > HQB_MAX_STAGES || needed > stage_count ||
      !geometry_ok(gm, &cb, &sc) || !to_raw_geo(gm, g))
    return HQB_ERR_INVALID;
  *st = RawStages{};
  for (uint32_t s = 0; s < needed; ++s) {
    if (stages[s].packed_codes == nullptr || stages[s].scales == nullptr || stages[s].packed_code_bytes != cb ||
        stages[s].scale_count != sc)
      return HQB_ERR_INVALID;
    st->codes[s] = stages[s].packed_codes;
    st->scales[s] = stages[s].scales;
  }
  return HQB_OK;
}

}  // namespace
}  // namespace hqb

using namespace hqb;

extern "C" {

HQB_API int hqb_raw_gemv(const hqb_geometry* gm, const hqb_raw_stage* stages, uint32_t stage_count, uint32_t prefix,
                         const float* x, uint64_t x_count, const float* bias, uint64_t bias_count, float* y,
                         uint64_t y_count, void* stream) {
  return hqb_raw_gemv_ex(gm, stages, stage_count, prefix, x, x_count, bias, bias_count, y, y_count, 0u, stream);
}

HQB_API int hqb_raw_gemv_ex(const hqb_geometry* gm, const hqb_raw_stage* stages, uint32_t stage_count,
                            uint32_t prefix, const float* x, uint64_t x_count, const float* bias,
                            uint64_t bias_count, float* y, uint64_t y_count, uint32_t flags, void* stream) {
  if (gm == nullptr || (stage_count > 0 && stages == nullptr)) return HQB_ERR_INVALID;
  if ((flags & ~(HQB_RAW_GENERIC | HQB_RAW_REQUIRE_FAST)) != 0 ||
      (flags & (HQB_RAW_GENERIC | HQB_RAW_REQUIRE_FAST)) == (HQB_RAW_GENERIC | HQB_RAW_REQUIRE_FAST))
    return HQB_ERR_INVALID;
  uint64_t cb = 0, sc = 0;
  if (!geometry_ok(gm, &cb, &sc) || stage_count == 0 || stage_count > HQB_MAX_STAGES || prefix > stage_count ||
      x == nullptr || x_count != gm->original_columns || y == nullptr || y_count != gm->original_rows ||
      ((bias == nullptr) != (bias_count == 0)) || (bias != nullptr && bias_count != gm->original_rows))
    return HQB_ERR_INVALID;
  RawGeo g{};
  if (!to_raw_geo(gm, &g)) return HQB_ERR_INVALID;
  RawStages st{};
  for (uint32_t s = 0; s < prefix; ++s) {
    if (stages[s].packed_codes == nullptr || stages[s].packed_code_bytes != cb || stages[s].scale_fp16_bits == nullptr ||
        stages[s].scale_count != sc)
      return HQB_ERR_INVALID;
    st.codes[s] = stages[s].packed_codes;
    st.scales[s] = stages[s].scale_fp16_bits;
  }
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  if (!(flags & HQB_RAW_GENERIC)) {
    RawI8Launch a{};
    a.geometry = gm;
    for (uint32_t s = 0; s < prefix; ++s) {
      a.codes[s] = stages[s].packed_codes;
      a.scales[s] = stages[s].scale_fp16_bits;
    }
    a.prefix = prefix;
    a.x = x;
    a.bias = bias;
    a.y = y;
    const int r = launch_raw_i8(a, stream);
    if (r != HQB_ERR_UNSUPPORTED || (flags & HQB_RAW_REQUIRE_FAST)) return r;
  }
  const unsigned blocks = grid_for(g.rows, 8);
  const bool bytes = (g.group % 4 == 0) && (g.padded_cols % 4 == 0);
  if (bytes) raw_gemv_kernel<true><<<blocks, 256, 0, as_stream(stream)>>>(g, st, prefix, x, bias, y);
  else raw_gemv_kernel<false><<<blocks, 256, 0, as_stream(stream)>>>(g, st, prefix, x, bias, y);
  return cudaGetLastError();
}

HQB_API int hqb_raw_dequantize_stage(const hqb_geometry* gm, const hqb_raw_stage_f32* stages, uint32_t stage_count,
                                     uint32_t stage, float* out, void* stream) {
  RawGeo g{};
  RawStages st{};
  if (out == nullptr || stage >= stage_count) return HQB_ERR_INVALID;
  const int rc = f32_stages(gm, stages, stage_count, stage + 1, &g, &st);
  if (rc != HQB_OK) return rc;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  raw_dequantize_kernel<<<grid_for(g.rows * g.cols, 256), 256, 0, as_stream(stream)>>>(g, st, stage, stage + 1, 0, out);
  return cudaGetLastError();
}

HQB_API int hqb_raw_dequantize_prefix(const hqb_geometry* gm, const hqb_raw_stage_f32* stages, uint32_t stage_count,
                                      uint32_t prefix, float* out, void* stream) {
  RawGeo g{};
  RawStages st{};
  if (out == nullptr || prefix > stage_count) return HQB_ERR_INVALID;
  const int rc = f32_stages(gm, stages, stage_count, prefix, &g, &st);
  if (rc != HQB_OK) return rc;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  raw_dequantize_kernel<<<grid_for(g.rows * g.cols, 256), 256, 0, as_stream(stream)>>>(g, st, 0, prefix, 1, out);
  return cudaGetLastError();
}

HQB_API int hqb_raw_linear_ordered(const hqb_geometry* gm, const hqb_raw_stage_f32* stages, uint32_t stage_count,
                                   uint32_t prefix, const float* x, uint64_t batch, const float* bias, float* y,
                                   void* stream) {
  RawGeo g{};
  RawStages st{};
  if (prefix > stage_count || (batch > 0 && (x == nullptr || y == nullptr))) return HQB_ERR_INVALID;
  const int rc = f32_stages(gm, stages, stage_count, prefix, &g, &st);
  if (rc != HQB_OK) return rc;
  if (batch == 0) return HQB_OK;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  raw_linear_ordered_kernel<<<grid_for(batch * g.rows, 128), 128, 0, as_stream(stream)>>>(g, st, prefix, x, batch, bias,
                                                                                          y);
  return cudaGetLastError();
}

}  // extern "C"
