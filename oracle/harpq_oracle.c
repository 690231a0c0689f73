/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle (plain C restatement) for the progressive
 * int2 GEMV path.  Never linked into the product library; tests/, smoke() and
 * bench.py's cpu_baseline leg use it as the checker.
 *
 * Each function cites the reference file:line whose behaviour it restates.
 * Built with -ffp-contract=off so that every FP32 multiply and add rounds
 * separately, as the reference's scalar loops do on x86-64 without FMA.
 */
#include "harpq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* CRC32C (Castagnoli, reflected polynomial 0x82F63B78), table-driven.
 * Restates native/src/stage_codec.cpp:147-157 and :328-339 (and
 * src/harpq/integrity.py:24-54). */
uint32_t hqo_crc32c(const uint8_t* data, size_t size, uint32_t crc) {
  static uint32_t table[256];
  static int ready = 0;
  if (!ready) {
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t v = i;
      for (int bit = 0; bit < 8; ++bit) {
        v = (v >> 1) ^ ((v & 1u) ? 0x82F63B78u : 0u);
      }
      table[i] = v;
    }
    ready = 1;
  }
  uint32_t value = crc ^ 0xFFFFFFFFu;
  for (size_t i = 0; i < size; ++i) {
    value = table[(value ^ data[i]) & 0xFFu] ^ (value >> 8);
  }
  return value ^ 0xFFFFFFFFu;
}

/* IEEE binary16 -> binary32, exact.  Restates stage_codec.cpp:46-63. */
float hqo_half_to_float(uint16_t half) {
  const uint32_t sign = (uint32_t)(half & 0x8000u) << 16;
  const uint32_t exponent = (half >> 10) & 0x1Fu;
  const uint32_t mantissa = half & 0x3FFu;
  float magnitude;
  if (exponent == 0) {
    magnitude = ldexpf((float)mantissa, -24); /* subnormal or zero */
  } else if (exponent == 0x1F) {
    magnitude = mantissa == 0 ? INFINITY : NAN;
  } else {
    magnitude = ldexpf(1.0f + (float)mantissa / 1024.0f, (int)exponent - 15);
  }
  float result = magnitude;
  if (sign) result = -result;
  return result;
}

/* Signed int2 code of element i: ((byte >> 2*(i%4)) & 3), values >= 2 wrap to
 * negative.  Restates stage_codec.cpp:139-145 (and quantization.py:63-91). */
int8_t hqo_decode_code(const uint8_t* packed_codes, uint64_t element_index) {
  const uint8_t packed = packed_codes[element_index / 4];
  const unsigned shift = (unsigned)((element_index % 4) * 2);
  const uint8_t raw = (uint8_t)((packed >> shift) & 0x03u);
  return (int8_t)(raw >= 2 ? (int)raw - 4 : (int)raw);
}

static uint16_t read_le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t read_le32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
         ((uint32_t)p[3] << 24);
}

/* HQSTAGE payload: "HQSTAGE\0", u16 version (1), u16 stage, u32 code bytes,
 * u32 scale count, codes, little-endian FP16 scales.  Validation order restates
 * stage_codec.cpp:161-216 (and matrix_codec.py:17-18, :120-151). */
int hqo_decode_payload(const uint8_t* payload, size_t payload_size,
                       uint16_t expected_stage, uint64_t expected_scale_count,
                       uint8_t* codes_out, uint64_t codes_cap, uint64_t* code_bytes,
                       float* scales_out, uint64_t scales_cap, uint64_t* scale_count) {
  static const uint8_t magic[8] = {'H', 'Q', 'S', 'T', 'A', 'G', 'E', 0};
  if (payload_size < 20) return HQO_ERR_TRUNCATED;
  if (memcmp(payload, magic, 8) != 0) return HQO_ERR_MAGIC;
  const uint16_t version = read_le16(payload + 8);
  const uint16_t stage = read_le16(payload + 10);
  const uint64_t ncodes = read_le32(payload + 12);
  const uint64_t nscales = read_le32(payload + 16);
  if (version != 1) return HQO_ERR_VERSION;
  if (stage != expected_stage) return HQO_ERR_STAGE;
  if (nscales != expected_scale_count) return HQO_ERR_SCALE_COUNT;
  if ((uint64_t)payload_size != 20 + ncodes + 2 * nscales) return HQO_ERR_LENGTH;
  if (ncodes > codes_cap || nscales > scales_cap) return HQO_ERR_CAPACITY;
  memcpy(codes_out, payload + 20, ncodes);
  const uint8_t* sp = payload + 20 + ncodes;
  for (uint64_t i = 0; i < nscales; ++i) {
    const float s = hqo_half_to_float(read_le16(sp + 2 * i));
    if (!isfinite(s)) return HQO_ERR_NONFINITE;
    if (s < 0.0f) return HQO_ERR_NEGATIVE;
    scales_out[i] = s;
  }
  *code_bytes = ncodes;
  *scale_count = nscales;
  return HQO_OK;
}

static uint64_t ceil_div(uint64_t a, uint64_t b) { return a / b + (a % b != 0); }

/* Restates ValidateMatrix, stage_codec.cpp:80-137.  Stage identity is implicit
 * (index order of the array). */
int hqo_validate(const hqo_geometry* g, const hqo_stage* stages, uint32_t stage_count) {
  if (g->original_rows == 0 || g->original_columns == 0) return HQO_ERR_GEOMETRY;
  if (g->tile_rows == 0 || g->tile_columns == 0 || g->group_size == 0) return HQO_ERR_GEOMETRY;
  if (g->tile_columns % g->group_size != 0) return HQO_ERR_GEOMETRY;
  if (g->padded_rows != ceil_div(g->original_rows, g->tile_rows) * g->tile_rows ||
      g->padded_columns != ceil_div(g->original_columns, g->tile_columns) * g->tile_columns)
    return HQO_ERR_GEOMETRY;
  if (stage_count == 0 || stage_count > 4) return HQO_ERR_GEOMETRY;
  const uint64_t code_bytes = ceil_div(g->padded_rows * g->padded_columns, 4);
  const uint64_t scale_count = (g->padded_rows / g->tile_rows) *
                               (g->padded_columns / g->tile_columns) * g->tile_rows *
                               (g->tile_columns / g->group_size);
  for (uint32_t s = 0; s < stage_count; ++s) {
    if (stages[s].packed_code_bytes != code_bytes || stages[s].scale_count != scale_count)
      return HQO_ERR_GEOMETRY;
    for (uint64_t i = 0; i < scale_count; ++i) {
      const float v = stages[s].scales[i];
      if (!isfinite(v) || v < 0.0f) return HQO_ERR_GEOMETRY;
    }
  }
  return HQO_OK;
}

/* Scale index of (row, column): [tile_row][tile_col][row_in_tile][group].
 * Restates stage_codec.cpp:231-244. */
static uint64_t scale_index(const hqo_geometry* g, uint64_t row, uint64_t col) {
  const uint64_t grid_c = g->padded_columns / g->tile_columns;
  const uint64_t groups = g->tile_columns / g->group_size;
  const uint64_t tr = row / g->tile_rows, rit = row % g->tile_rows;
  const uint64_t tc = col / g->tile_columns;
  const uint64_t grp = (col % g->tile_columns) / g->group_size;
  return ((tr * grid_c + tc) * g->tile_rows + rit) * groups + grp;
}

static float stage_weight(const hqo_geometry* g, const hqo_stage* st, uint64_t row, uint64_t col) {
  const uint64_t code_index = row * g->padded_columns + col;
  return (float)hqo_decode_code(st->packed_codes, code_index) * st->scales[scale_index(g, row, col)];
}

/* Restates DequantizeStage, stage_codec.cpp:218-252. */
int hqo_dequantize_stage(const hqo_geometry* g, const hqo_stage* stages,
                         uint32_t stage_count, uint32_t stage_index, float* out) {
  int rc = hqo_validate(g, stages, stage_count);
  if (rc) return rc;
  if (stage_index >= stage_count) return HQO_ERR_PREFIX;
  for (uint64_t r = 0; r < g->original_rows; ++r)
    for (uint64_t c = 0; c < g->original_columns; ++c)
      out[r * g->original_columns + c] = stage_weight(g, &stages[stage_index], r, c);
  return HQO_OK;
}

/* Restates DequantizePrefix, stage_codec.cpp:254-272: stage matrices are added
 * in stage order into a 0.0f-initialised FP32 buffer. */
int hqo_dequantize_prefix(const hqo_geometry* g, const hqo_stage* stages,
                          uint32_t stage_count, uint32_t prefix, float* out) {
  int rc = hqo_validate(g, stages, stage_count);
  if (rc) return rc;
  if (prefix > stage_count) return HQO_ERR_PREFIX;
  const uint64_t n = g->original_rows * g->original_columns;
  for (uint64_t i = 0; i < n; ++i) out[i] = 0.0f;
  for (uint32_t s = 0; s < prefix; ++s)
    for (uint64_t r = 0; r < g->original_rows; ++r)
      for (uint64_t c = 0; c < g->original_columns; ++c)
        out[r * g->original_columns + c] += stage_weight(g, &stages[s], r, c);
  return HQO_OK;
}

static int tile_depth(const hqo_geometry* g, const uint8_t* depth, uint64_t row, uint64_t col) {
  const uint64_t grid_c = g->padded_columns / g->tile_columns;
  return depth[(row / g->tile_rows) * grid_c + col / g->tile_columns];
}

static int check_depth(const hqo_geometry* g, const uint8_t* depth, uint32_t stage_count) {
  const uint64_t tiles = (g->padded_rows / g->tile_rows) * (g->padded_columns / g->tile_columns);
  for (uint64_t t = 0; t < tiles; ++t)
    if (depth[t] > stage_count) return HQO_ERR_PREFIX;
  return HQO_OK;
}

/* Mixed-depth decode: same stage-ordered sum as DequantizePrefix, restricted per
 * tile (no reference symbol; the allocator's per-group prefix, allocator.py:1-9). */
int hqo_dequantize_mixed(const hqo_geometry* g, const hqo_stage* stages,
                         uint32_t stage_count, const uint8_t* depth, float* out) {
  int rc = hqo_validate(g, stages, stage_count);
  if (rc) return rc;
  if ((rc = check_depth(g, depth, stage_count))) return rc;
  const uint64_t n = g->original_rows * g->original_columns;
  for (uint64_t i = 0; i < n; ++i) out[i] = 0.0f;
  for (uint32_t s = 0; s < stage_count; ++s)
    for (uint64_t r = 0; r < g->original_rows; ++r)
      for (uint64_t c = 0; c < g->original_columns; ++c)
        if ((int)s < tile_depth(g, depth, r, c))
          out[r * g->original_columns + c] += stage_weight(g, &stages[s], r, c);
  return HQO_OK;
}

static int check_inputs(const hqo_geometry* g, const float* inputs, uint64_t batch,
                        const float* bias) {
  for (uint64_t i = 0; i < batch * g->original_columns; ++i)
    if (!isfinite(inputs[i])) return HQO_ERR_INPUT;
  if (bias)
    for (uint64_t i = 0; i < g->original_rows; ++i)
      if (!isfinite(bias[i])) return HQO_ERR_INPUT;
  return HQO_OK;
}

/* Shared scalar loop of ProgressiveLinearReference, stage_codec.cpp:302-324:
 * per stage, a fresh FP32 dot per (batch,row) summed column by column, added to
 * the output; bias added once at the end. */
static void linear_scalar(const hqo_geometry* g, const hqo_stage* stages,
                          uint32_t stage_count, uint32_t prefix, const uint8_t* depth,
                          const float* inputs, uint64_t batch, const float* bias,
                          float* out) {
  const uint64_t rows = g->original_rows, cols = g->original_columns;
  float* w = (float*)malloc(sizeof(float) * (cols ? cols : 1));
  for (uint64_t i = 0; i < batch * rows; ++i) out[i] = 0.0f;
  const uint32_t stop = depth ? stage_count : prefix;
  for (uint32_t s = 0; s < stop; ++s) {
    for (uint64_t r = 0; r < rows; ++r) {
      for (uint64_t c = 0; c < cols; ++c) {
        const int use = depth ? ((int)s < tile_depth(g, depth, r, c)) : 1;
        w[c] = use ? stage_weight(g, &stages[s], r, c) : 0.0f;
      }
      for (uint64_t b = 0; b < batch; ++b) {
        float dot = 0.0f;
        for (uint64_t c = 0; c < cols; ++c) dot += inputs[b * cols + c] * w[c];
        out[b * rows + r] += dot;
      }
    }
  }
  if (bias)
    for (uint64_t b = 0; b < batch; ++b)
      for (uint64_t r = 0; r < rows; ++r) out[b * rows + r] += bias[r];
  free(w);
}

/* Restates ProgressiveLinearReference, stage_codec.cpp:274-326. */
int hqo_linear_reference(const hqo_geometry* g, const hqo_stage* stages,
                         uint32_t stage_count, uint32_t prefix,
                         const float* inputs, uint64_t batch, const float* bias,
                         float* out) {
  int rc = hqo_validate(g, stages, stage_count);
  if (rc) return rc;
  if (prefix > stage_count) return HQO_ERR_PREFIX;
  if ((rc = check_inputs(g, inputs, batch, bias))) return rc;
  linear_scalar(g, stages, stage_count, prefix, NULL, inputs, batch, bias, out);
  return HQO_OK;
}

int hqo_linear_mixed(const hqo_geometry* g, const hqo_stage* stages,
                     uint32_t stage_count, const uint8_t* depth,
                     const float* inputs, uint64_t batch, const float* bias,
                     float* out) {
  int rc = hqo_validate(g, stages, stage_count);
  if (rc) return rc;
  if ((rc = check_depth(g, depth, stage_count))) return rc;
  if ((rc = check_inputs(g, inputs, batch, bias))) return rc;
  linear_scalar(g, stages, stage_count, stage_count, depth, inputs, batch, bias, out);
  return HQO_OK;
}
