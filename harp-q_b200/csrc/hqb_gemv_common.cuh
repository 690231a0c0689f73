// Device code shared by the plane-layout GEMV kernels (hqb_plane.cu, hqb_bulk.cu):
// launch parameters, activation preparation (FP16 fragments and int8 limbs), output
// stores, split-tile-row publication and reduction, resident activation slots, the
// int8-limb tensor-core tile step and the per-tile depth-map range search.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "harpq_b200.h"
#include "hqb_device.cuh"
#include "hqb_schedule.h"

namespace hqb {

constexpr uint32_t kRowBlockBytes = 544;
constexpr uint32_t kRecordBytes = HQB_TILE_RECORD_BYTES;
constexpr uint32_t kConsumerWarps = 8;
constexpr uint32_t kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kUnitsInFlight = 12;     // tile-stages buffered per CTA (52 KB)
constexpr uint32_t kSmemBudget = 100 * 1024;  // ring bytes per CTA, two CTAs per SM
constexpr uint32_t kMaxCtasPerSm = 4;  // bound on resident CTAs per SM (sizes the partials)

static_assert(kRecordBytes == 8 * kRowBlockBytes, "record = 8 row blocks");

struct GemvParams {
  const uint8_t* planes[HQB_MAX_STAGES];
  const uint8_t* depth;  // [R][C] or null (uniform)
  const uint32_t* plan;  // [R+1] or null
  const uint8_t* xfrag;
  const void* x_raw;   // raw activations [batch][cols] when the GEMV prepares them itself
  const void* bias;
  void* y;
  float* partials;     // [G][2][batch][128]
  uint32_t* counters;  // [R] split-row arrival counts (zero between launches)
  int* error;
  uint64_t total;      // units (uniform); mixed reads plan[R]
  uint32_t rows;
  uint32_t R, C;
  uint32_t prefix;
  uint32_t stage_count;
  uint32_t batch;
  uint32_t xslot_bytes;
  uint32_t ring_slots;   // ring slots (runs) per CTA
  uint32_t slot_stride;  // header + activation fragments + max-run records
  uint32_t shift_mul;    // 2^24: w >> 8 computed as a high multiply
  uint32_t pdl;          // launched as a programmatic dependent
  uint32_t x_resident;   // all activation fragments staged once per CTA (else one per slot)
  uint32_t slot_x_bytes; // activation bytes carried by each slot (0 when resident)
  uint32_t cols;         // original columns (raw activation rows)
  // fused all-gather (g_world > 1): outputs go to every rank's gathered buffer
  uint32_t g_world, g_rank;
  uint64_t g_slot_rows;
  void* g_peer_y[HQB_MAX_PEERS];
  uint32_t* g_peer_flags[HQB_MAX_PEERS];
  uint32_t* g_done;      // CTAs of this launch that finished (local, returns to zero)
  uint32_t x_vec;        // raw activation rows can be read as aligned 16-byte chunks
  uint32_t xw_bytes;     // row-block kernel: fragment bytes of each warp's shared-memory area
  uint32_t x_res_slots;  // uniform stream-K kernel: resident activation slots per CTA
  uint32_t chunk_tiles;  // bulk-copy kernel: walk tiles per ring chunk
  int bias_dtype;
  int y_dtype;
};

__host__ __device__ inline uint32_t xslot_bytes_for(uint32_t batch, uint32_t xl) {
  return static_cast<uint32_t>((batch * (256u * xl + 8u) + 15u) / 16u * 16u);
}

constexpr int kPrefetch = 4;
constexpr uint32_t kStreamThreads = kConsumerWarps * 32;

// --------------------------------------------------------------------------------------
// activation preparation

// 2^k as a float for -126 <= k <= 127 (normal range), from the IEEE-754 bit layout.
__device__ __forceinline__ float exp2_int(int k) { return __int_as_float((k + 127) << 23); }

// Four consecutive activations [col0, col0 + 4) of one row as FP32, zero past `cols`.
// vec: the row start is 16-byte aligned and cols is a multiple of 16 bytes of elements,
// so the four lie wholly inside or wholly outside the row and load as one vector.
template <typename XT>
__device__ __forceinline__ void load_x4(const XT* row, uint32_t col0, uint32_t cols, bool vec, float (&v)[4]) {
  if (vec) {
    if (col0 >= cols) {
      v[0] = v[1] = v[2] = v[3] = 0.0f;
    } else if constexpr (sizeof(XT) == 2) {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(row + col0));
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[0] = f0.x;
      v[1] = f0.y;
      v[2] = f1.x;
      v[3] = f1.y;
    } else {
      const float4 f = __ldcg(reinterpret_cast<const float4*>(row + col0));
      v[0] = f.x;
      v[1] = f.y;
      v[2] = f.z;
      v[3] = f.w;
    }
    return;
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float f = 0.0f;
    if (col0 + t < cols) {
      if constexpr (sizeof(XT) == 2) f = __half2float(row[col0 + t]);
      else f = row[col0 + t];
    }
    v[t] = f;
  }
}

// Preparation of W (tile column, batch row) items, one warp per item; lane L holds
// columns 4L..4L+3 of the item's tile (v, zero past the last column).  Per item:
//   e    tile exponent: the largest |x| of the tile lands in [2^14, 2^15) after 2^-e;
//   the B fragments: FP16 x·2^-e·4^-(c%4) of column c at half (4b + c/32)·32 + (c%8)·4
//        + (c%32)/8 of the slot (XL 2: the FP16 remainder batch·256 bytes further on);
//   {2^(24+e), 2^(e+1)·Σ_c x̃_c·4^(c%4)} at byte batch·256·XL + 8b, x̃ the stored value.
// The sum adds each lane's four terms pairwise, then across lanes in butterfly order.
// Every preparation path (prep_x_kernel and both in-kernel paths) goes through this
// function, so their fragments are bit-identical.
template <int XL, int W>
__device__ __forceinline__ void prep_items(const float (&v)[W][4], const bool (&ok)[W], uint8_t* const (&slot)[W],
                                           const uint32_t (&b)[W], uint32_t batch, uint32_t lane) {
  float a[W];
#pragma unroll
  for (int w = 0; w < W; ++w)
    a[w] = fmaxf(fmaxf(fabsf(v[w][0]), fabsf(v[w][1])), fmaxf(fabsf(v[w][2]), fabsf(v[w][3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int w = 0; w < W; ++w) a[w] = fmaxf(a[w], __shfl_xor_sync(0xffffffffu, a[w], o));
  // column 4L + t: quad L/8, position m = 4(L%2) + t, column group (L%8)/2
  const uint32_t pos = 32 * (lane >> 3) + 16 * (lane & 1) + ((lane & 7) >> 1);
  int e[W];
  float s[W];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    // |x| >= 2^-24 is a normal float, so the biased exponent field gives floor(log2)
    e[w] = a[w] > 0.0f ? max(-100, min(100, ((__float_as_int(a[w]) >> 23) & 0xff) - 127 - 14)) : 0;
    __half* dst = reinterpret_cast<__half*>(slot[w]) + b[w] * 128 + pos;
    float part[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float xs = v[w][t] * exp2_int(-e[w] - 2 * t);
      const __half hi = __float2half_rn(xs);
      float eff = __half2float(hi);
      if (ok[w]) dst[4 * t] = hi;
      if constexpr (XL == 2) {
        const __half lo = __float2half_rn(xs - eff);
        eff += __half2float(lo);
        if (ok[w]) dst[batch * 128 + 4 * t] = lo;
      }
      part[t] = eff * exp2_int(2 * t);
    }
    s[w] = (part[0] + part[1]) + (part[2] + part[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int w = 0; w < W; ++w) s[w] += __shfl_xor_sync(0xffffffffu, s[w], o);
  if (lane == 0) {
#pragma unroll
    for (int w = 0; w < W; ++w)
      if (ok[w])
        *reinterpret_cast<float2*>(slot[w] + batch * 256 * XL + b[w] * 8) =
            make_float2(exp2_int(24 + e[w]), s[w] * exp2_int(e[w] + 1));
  }
}

// ---- int8 activation limbs (FP16 or FP32 x, batch <= 2) ------------------------------
//
// The integer tensor-core path multiplies u8 code fragments by s8 activation limbs with
// m16n8k32 (exact s32 accumulate).  One AND with 0x03030303 << 2m turns a plane code
// word into an A register whose byte j holds (code+2)·4^m of column 4j+m of the word's
// 16 columns, so MMA m of a row block reads code position m of every byte, and its
// B operand carries Y = round(x·2^(30-E-2m)) for those columns: the factor 4^m cancels
// and every product is (code+2)·x·2^(30-E) up to the rounding of x.  E is the tile's
// exponent (max|x| < 2^E), so |Y| <= 2^30 and x keeps at least 24 significant bits
// relative to the tile maximum (an FP16 x is exact down to 2^-13 of it).  Y splits into
// four balanced signed bytes Y = Σ_l limb_l·2^(24-8l).  The limbs ride in the MMA's N
// columns: column n = 2·limb + batch row, so one MMA serves batch 1 and 2 alike.  An
// accumulator that starts from the bits of 1.5·2^23 reads, as FP32, 1.5·2^23 +
// Σ(code+2)·limb (|Σ| < 2^21), so one FMA with the column's {L, K} =
// {2^(E-6-8·limb), -(1.5·2^23 + 2·Σlimb)·L} gives the exact limb sum Σcode·limb·L.
//
// Slot of one tile (xslot_i8_bytes): entries e = limb·batch + b of 128 bytes, 32 per
// lane quad position q, word 2m + h of which is the B register b_h of MMA m (bytes j:
// column 32q + 16h + 4j + m); then 8 columns × {L, K} FP32 ({0, 0} for columns no
// limb uses).
constexpr uint32_t kLimbs = 4;
constexpr uint32_t kAccBiasBits = 0x4B400000u;  // FP32 1.5·2^23
constexpr float kAccBias = 12582912.0f;

// Slot bytes: the limb entries, 8 accumulator columns x {L, K}, and 16 bytes holding each
// batch row's wide-tile factor (limb_item).
__host__ __device__ inline uint32_t xslot_i8_bytes(uint32_t batch) { return kLimbs * batch * 128u + 80u; }
constexpr uint32_t kLimbMaxE = 100;  // tiles with max|x| >= 2^100 carry a wide factor

// Limb preparation of W (tile column, batch row) items, one warp per item; lane L holds
// columns 4L..4L+3 of the item's tile (v, zero past the last column).  The row-block
// kernel (gemv_rows_kernel) builds its slots here; limb_item, with another lane layout,
// builds the same bytes (for every finite tile below 2^kLimbMaxE) for the stream-K,
// grouped, bulk and raw kernels.
template <int W>
__device__ __forceinline__ void prep_i8_items(const float (&v)[W][4], const bool (&ok)[W], uint8_t* const (&slot)[W],
                                              const uint32_t (&b)[W], uint32_t batch, uint32_t lane) {
  float a[W];
#pragma unroll
  for (int w = 0; w < W; ++w)
    a[w] = fmaxf(fmaxf(fabsf(v[w][0]), fabsf(v[w][1])), fmaxf(fabsf(v[w][2]), fabsf(v[w][3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int w = 0; w < W; ++w) a[w] = fmaxf(a[w], __shfl_xor_sync(0xffffffffu, a[w], o));
  // A tile holding a NaN or an Inf, or a value of 2^100 or more (beyond this form's limb
  // factors), gets NaN constants: every output of its batch row is NaN rather than wrong.
  // (The bulk kernel's limb_item keeps such finite values exact.)
  bool bad[W];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const bool lane_bad = !(isfinite(v[w][0]) && isfinite(v[w][1]) && isfinite(v[w][2]) && isfinite(v[w][3])) ||
                          a[w] >= 1.2676506e30f;  // 2^100
    bad[w] = __any_sync(0xffffffffu, lane_bad);
  }
  int E[W], sum[W][kLimbs];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    // a < 2^E: the biased exponent field of a normal float gives floor(log2 a); the
    // clamp keeps every limb factor 2^(E-6-8l) a normal float
    E[w] = a[w] > 0.0f && !bad[w] ? max(-90, min(100, ((__float_as_int(a[w]) >> 23) & 0xff) - 126)) : 0;
    // column 4L + t: quad position L/8, half (L%8)/4, byte L%4 of word 2t + half
    uint8_t* base = slot[w] + (lane >> 3) * 32 + (lane & 7);
#pragma unroll
    for (int l = 0; l < static_cast<int>(kLimbs); ++l) sum[w][l] = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      int y = __float2int_rn(v[w][t] * exp2_int(30 - E[w] - 2 * t));
      int limb[kLimbs];
#pragma unroll
      for (int l = static_cast<int>(kLimbs) - 1; l > 0; --l) {
        limb[l] = (y << 24) >> 24;  // balanced low byte
        y = (y - limb[l]) >> 8;
      }
      limb[0] = y;  // |limb 0| <= 64
#pragma unroll
      for (int l = 0; l < static_cast<int>(kLimbs); ++l) {
        if (ok[w]) base[(l * batch + b[w]) * 128 + 8 * t] = static_cast<uint8_t>(limb[l] & 0xff);
        sum[w][l] += limb[l] * (1 << (2 * t));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int w = 0; w < W; ++w)
#pragma unroll
      for (int l = 0; l < static_cast<int>(kLimbs); ++l) sum[w][l] += __shfl_xor_sync(0xffffffffu, sum[w][l], o);
  if (lane == 0) {
#pragma unroll
    for (int w = 0; w < W; ++w) {
      if (!ok[w]) continue;
      float* cst = reinterpret_cast<float*>(slot[w] + kLimbs * batch * 128);
#pragma unroll
      for (int l = 0; l < static_cast<int>(kLimbs); ++l) {
        const uint32_t n = 2 * l + b[w];
        const float L = exp2_int(E[w] - 6 - 8 * l);
        cst[2 * n] = bad[w] ? __uint_as_float(0x7fc00000u) : L;
        cst[2 * n + 1] = bad[w] ? __uint_as_float(0x7fc00000u) : -(kAccBias + static_cast<float>(2 * sum[w][l])) * L;
      }
      if (b[w] == 0) {
        for (uint32_t n = 0; n < 8; ++n)
          if (n >= 2 * kLimbs || (batch == 1 && (n & 1))) cst[2 * n] = cst[2 * n + 1] = 0.0f;
      }
    }
  }
}

// One (tile column c, batch row b) item of an int8 limb slot, built by one warp with one
// 32-bit store per lane and limb.  Lane L builds word L of every limb entry, i.e. the bytes
// of columns 32q + 16h + m + 4j (q = L/8, m = (L/2)%4, h = L%2, j = 0..3): the same slot,
// byte for byte, as prep_i8_items for every tile whose largest |x| is finite and below
// 2^kLimbMaxE.  Per lane:
//   Y_j = round(x_j·2^(30-E-2m)) (one scale: m is the lane's), and the balanced base-256
//   digits of Y_j are the bytes of (Y_j + 0x80808080) ^ 0x80808080; a byte transpose of the
//   four values gives the four limb words; each limb's Σ digit·4^m over the tile is one
//   dp4a per lane and one warp reduction.
// Tiles outside the fast representation:
//   * a NaN or Inf activation: {L, K} = NaN, so every output of that batch row is NaN;
//   * max|x| >= 2^kLimbMaxE (finite): the limbs keep x·2^(30-E-2m), L is divided by
//     2^(E-kLimbMaxE) so that K stays finite, K is stored negated (K >= 0 marks the tile),
//     and that factor is the row's wide factor at byte kLimbs·batch·128 + 64 + 4b of the
//     slot (1.0 otherwise); kernels that read it multiply the tile's stage sums by it.
// This lane's four activations of item (tile column c) for limb_item: columns
// 32q + 16h + m + 4j of the tile (zero past the last column).
template <typename XT>
__device__ __forceinline__ void limb_load(const XT* __restrict__ xrow, uint32_t c, uint32_t cols, uint32_t lane,
                                          float (&v)[4]) {
  const uint32_t q = lane >> 3, m = (lane >> 1) & 3u, h = lane & 1u;
  const uint32_t col0 = c * 128u + 32u * q + 16u * h + m;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t col = col0 + 4u * j;
    float f = 0.0f;
    if (col < cols) {
      if constexpr (sizeof(XT) == 2) f = __half2float(xrow[col]);
      else f = xrow[col];
    }
    v[j] = f;
  }
}

// The slot item from this lane's four activations (limb_load).
__device__ __forceinline__ void limb_item(const float (&v)[4], uint8_t* slot, uint32_t b, uint32_t batch,
                                          uint32_t lane) {
  const uint32_t m = (lane >> 1) & 3u;
  // the tile's largest |x| as FP32 bits: non-negative floats order as integers, and NaN
  // sorts above Inf
  uint32_t ab = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) ab = max(ab, __float_as_uint(v[j]) & 0x7fffffffu);
  ab = __reduce_max_sync(0xffffffffu, ab);
  const bool special = ab >= 0x7f800000u;
  // max|x| < 2^E from the exponent field; subnormal tiles take -90 (the limb factors stay
  // normal floats), an all-zero tile 0
  int E = ab == 0 ? 0 : max(-90, static_cast<int>(ab >> 23) - 126);
  if (special) E = 0;
  const int wide = E > static_cast<int>(kLimbMaxE) ? E - static_cast<int>(kLimbMaxE) : 0;
  const float scale = exp2_int(30 - E - 2 * static_cast<int>(m));
  uint32_t d[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int y = special ? 0 : __float2int_rn(v[j] * scale);
    d[j] = (static_cast<uint32_t>(y) + 0x80808080u) ^ 0x80808080u;  // balanced digits, limb 3 in byte 0
  }
  // byte transpose: word for limb l holds byte (3 - l) of d[0..3]
  const uint32_t t0 = __byte_perm(d[0], d[1], 0x5140), t1 = __byte_perm(d[2], d[3], 0x5140);
  const uint32_t t2 = __byte_perm(d[0], d[1], 0x7362), t3 = __byte_perm(d[2], d[3], 0x7362);
  const uint32_t wl[4] = {__byte_perm(t2, t3, 0x7632), __byte_perm(t2, t3, 0x5410), __byte_perm(t0, t1, 0x7632),
                          __byte_perm(t0, t1, 0x5410)};
  int sum[kLimbs];
#pragma unroll
  for (int l = 0; l < static_cast<int>(kLimbs); ++l) {
    *reinterpret_cast<uint32_t*>(slot + (l * batch + b) * 128u + lane * 4u) = wl[l];
    sum[l] = __reduce_add_sync(0xffffffffu, __dp4a(static_cast<int>(wl[l]), 0x01010101, 0) << (2 * m));
  }
  // {L, K} of accumulator column n = 2l + b: lane l < kLimbs; with batch 1 lanes 4..7 clear
  // the odd columns no limb uses
  float* cst = reinterpret_cast<float*>(slot + kLimbs * batch * 128u);
  if (lane < kLimbs) {
    const int l = static_cast<int>(lane);
    const int sl = l == 0 ? sum[0] : (l == 1 ? sum[1] : (l == 2 ? sum[2] : sum[3]));
    float L = exp2_int(E - wide - 6 - 8 * l);
    float K = -(kAccBias + static_cast<float>(2 * sl)) * L;
    if (wide) K = -K;  // K >= 0 marks a wide tile
    if (special) L = K = __uint_as_float(0x7fc00000u);
    *reinterpret_cast<float2*>(cst + 2 * (2 * lane + b)) = make_float2(L, K);
  } else if (lane < 2 * kLimbs && batch == 1) {
    *reinterpret_cast<float2*>(cst + 2 * (2 * (lane - kLimbs) + 1)) = make_float2(0.0f, 0.0f);
  } else if (lane == 2 * kLimbs) {
    cst[16 + b] = exp2_int(wide);  // the row's wide factor
  }
}


// Output element (batch b, row): local y, or with the fused gather every rank's gathered
// buffer [batch][world * slot_rows] at column rank * slot_rows + row (P2P stores).
__device__ __forceinline__ void put_y(const GemvParams& p, uint32_t b, uint32_t row, float v) {
  if (p.g_world > 1) {
    const uint64_t o = static_cast<uint64_t>(b) * p.g_world * p.g_slot_rows + p.g_rank * p.g_slot_rows + row;
    for (uint32_t r = 0; r < p.g_world; ++r) {
      if (p.y_dtype == HQB_F16) static_cast<__half*>(p.g_peer_y[r])[o] = __float2half_rn(v);
      else static_cast<float*>(p.g_peer_y[r])[o] = v;
    }
    return;
  }
  const uint64_t o = static_cast<uint64_t>(b) * p.rows + row;
  if (p.y_dtype == HQB_F16) static_cast<__half*>(p.y)[o] = __float2half_rn(v);
  else static_cast<float*>(p.y)[o] = v;
}

template <int NB>
__device__ __forceinline__ void store_out(const GemvParams& p, const float (&v)[NB][4], uint32_t row0,
                                          uint32_t q) {
  const uint32_t row1 = row0 + 8;
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t b = 2 * q + j + 8 * nb;
      if (b >= p.batch) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t row = h ? row1 : row0;
        if (row >= p.rows) continue;
        float out = v[nb][2 * h + j];
        if (p.bias != nullptr) {
          out += p.bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(p.bias)[row])
                                         : static_cast<const float*>(p.bias)[row];
        }
        put_y(p, b, row, out);
      }
    }
  }
}

struct RowSplit {
  uint32_t first, last;  // CTAs contributing to the tile row
};

__device__ __forceinline__ RowSplit row_split(const GemvParams& p, uint32_t r, uint64_t total, uint32_t ctas) {
  const uint64_t per_row = static_cast<uint64_t>(p.C) * p.prefix;
  const uint64_t rb = row_begin(r, p.plan, per_row), re = row_begin(r + 1, p.plan, per_row);
  return RowSplit{unit_owner(rb, total, ctas), unit_owner(re - 1, total, ctas)};
}

template <int NB>
__device__ __forceinline__ void publish_partial(const GemvParams& p, uint32_t cta, uint32_t k, const float (&y)[NB][4],
                                                uint32_t rit0, uint32_t q) {
  float* part = p.partials + static_cast<uint64_t>(cta * 2 + k) * p.batch * 128;
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t b = 2 * q + j + 8 * nb;
      if (b < p.batch) {
        part[b * 128 + rit0] = y[nb][j];
        part[b * 128 + rit0 + 8] = y[nb][2 + j];
      }
    }
}

// Accumulator chains per tile: one per stage; depth 1 alternates two chains.
template <int D>
struct TileChains {
  static constexpr int value = D == 1 ? 2 : D;
};

// A CTA's part of the split tile rows it touches: at most its first and its last row.
struct SplitRows {
  uint32_t row0, row1;
  uint32_t count;
};

// Split tile rows of the uniform stream-K kernel.  A CTA's part of a tile row that goes
// on in later CTAs is published as 64-bit words {FP32 bits, kPartFlag} in the CTA's one
// slot [cta][batch][128] of the partials region: one single-copy-atomic store per value,
// so no fence is needed.  The row's last contributor (the CTA in whose range it ends)
// waits (bounded) for the words of the earlier contributors, adds them in CTA order and
// its own part last, stores the rows and clears the words to zero.  Earlier CTAs never
// wait for later ones, so the scheme needs no co-residency beyond CTA-index order.  The
// partials region is all zero between launches (every consumer clears what it reads).
constexpr uint32_t kPartFlag = 0x7fc0a5a5u;  // an FP32 NaN pattern no arithmetic produces

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* a, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

template <int NB>
__device__ __forceinline__ void publish_flagged(const GemvParams& p, uint32_t cta, const float (&y)[NB][4],
                                                uint32_t rit0, uint32_t q) {
  unsigned long long* part = reinterpret_cast<unsigned long long*>(p.partials) + static_cast<uint64_t>(cta) * p.batch * 128;
  const unsigned long long flag = static_cast<unsigned long long>(kPartFlag) << 32;
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t b = 2 * q + j + 8 * nb;
      if (b < p.batch) {
        st_relaxed_gpu_u64(part + b * 128 + rit0, flag | __float_as_uint(y[nb][j]));
        st_relaxed_gpu_u64(part + b * 128 + rit0 + 8, flag | __float_as_uint(y[nb][2 + j]));
      }
    }
}

// Row r ends in this CTA (the last contributor): add the earlier contributors' parts in
// CTA order, then this warp's own part, plus bias, and store its rows.  The lane's
// elements (batch columns 2q + j, rows rit0 and rit0 + 8; with B1 only column 0) are
// gathered together: all loads of a group of contributors are issued at once, and the
// words not yet published are read again together (bounded), so waiting costs one
// round trip to L2 per round, not one per word.  Consumed words are cleared to zero.
template <int NB, bool B1>
__device__ __forceinline__ void reduce_split_row(const GemvParams& p, uint32_t r, uint64_t row_first_unit,
                                                 uint64_t total, uint32_t ctas, uint32_t cta,
                                                 const float (&own)[NB][4], uint32_t rit0, uint32_t q) {
  constexpr int J = B1 ? 1 : 2;                  // batch columns per lane and accumulator block
  constexpr int E = NB * J * 2;                  // elements per lane
  constexpr uint32_t K = E <= 2 ? 8 : (E <= 4 ? 4 : 2);  // contributors per group (16 words)
  const uint32_t first = unit_owner(row_first_unit, total, ctas);
  unsigned long long* part = reinterpret_cast<unsigned long long*>(p.partials);
  uint64_t off[E];
  bool ok[E];
  float sum[E];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = (nb * J + j) * 2 + h;
        const uint32_t b = 2 * q + j + 8 * nb;
        ok[e] = b < p.batch && (!B1 || q == 0);
        off[e] = static_cast<uint64_t>(ok[e] ? b : 0u) * 128 + rit0 + 8 * h;
        sum[e] = 0.0f;
      }
  bool gave_up = false;
  const uint64_t cta_words = static_cast<uint64_t>(p.batch) * 128;
  for (uint32_t i0 = first; i0 < cta; i0 += K) {
    unsigned long long v[K][E];
    const unsigned long long ready = static_cast<unsigned long long>(kPartFlag) << 32;
#pragma unroll
    for (uint32_t k = 0; k < K; ++k)
#pragma unroll
      for (int e = 0; e < E; ++e)
        v[k][e] = (i0 + k < cta && ok[e]) ? ld_relaxed_gpu_u64(part + (i0 + k) * cta_words + off[e]) : ready;
    unsigned long long t0 = 0;
    for (;;) {
      bool all = true;
#pragma unroll
      for (uint32_t k = 0; k < K; ++k)
#pragma unroll
        for (int e = 0; e < E; ++e) all = all && (v[k][e] >> 32) == kPartFlag;
      if (all || gave_up) break;
      if (t0 == 0) {
        t0 = global_timer_ns();
      } else if (global_timer_ns() - t0 > kWaitLimitNs) {
        atomicOr(p.error, HQB_DEVERR_TIMEOUT);
        gave_up = true;
        break;
      }
#pragma unroll
      for (uint32_t k = 0; k < K; ++k)
#pragma unroll
        for (int e = 0; e < E; ++e)
          if ((v[k][e] >> 32) != kPartFlag) v[k][e] = ld_relaxed_gpu_u64(part + (i0 + k) * cta_words + off[e]);
    }
#pragma unroll
    for (uint32_t k = 0; k < K; ++k)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (i0 + k < cta && ok[e]) {
          sum[e] += __uint_as_float(static_cast<uint32_t>(v[k][e]));
          st_relaxed_gpu_u64(part + (i0 + k) * cta_words + off[e], 0ull);
        }
  }
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = (nb * J + j) * 2 + h;
        const uint32_t b = 2 * q + j + 8 * nb, row = r * 128 + rit0 + 8 * h;
        if (!ok[e] || row >= p.rows) continue;
        float y = sum[e] + own[nb][2 * h + j];
        if (p.bias != nullptr)
          y += p.bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(p.bias)[row])
                                       : static_cast<const float*>(p.bias)[row];
        put_y(p, b, row, y);
      }
}

// After the CTA's last tile: one barrier, then one arrival per split row on a per-row
// counter (acquire-release atomics issued together by one thread; the barrier orders
// every thread's published part before that thread's release).  The contributor that
// arrives last resets the counter and sums the parts of all contributors in CTA order
// plus bias (the arithmetic of fixup_kernel), reading them through L2.  Nothing waits
// on another CTA.
template <int NB>
__device__ __forceinline__ void finish_split_rows(const GemvParams& p, const SplitRows& split,
                                                  uint64_t units_per_row, uint64_t total, uint32_t ctas,
                                                  uint32_t* s_info, uint32_t nthreads = kStreamThreads) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t r0 = split.row0, r1 = split.row1;
    const uint32_t old0 = atom_add_acq_rel_gpu(p.counters + r0, 1u);
    const uint32_t old1 = split.count > 1 ? atom_add_acq_rel_gpu(p.counters + r1, 1u) : 0u;
    uint32_t n = 0;
#pragma unroll
    for (uint32_t i = 0; i < 2; ++i) {
      if (i >= split.count) break;
      const uint32_t r = i == 0 ? r0 : r1;
      const uint64_t rb = static_cast<uint64_t>(r) * units_per_row, re = rb + units_per_row;
      const uint32_t first = unit_owner(rb, total, ctas), last = unit_owner(re - 1, total, ctas);
      if ((i == 0 ? old0 : old1) == last - first) {  // every other contributor has published
        p.counters[r] = 0u;                           // ready for the next launch
        s_info[1 + 4 * n] = r;
        s_info[2 + 4 * n] = first;
        s_info[3 + 4 * n] = last;
        s_info[4 + 4 * n] = unit_start(first, total, ctas) < rb ? 1u : 0u;
        ++n;
      }
    }
    s_info[0] = n;
  }
  __syncthreads();
  const uint32_t n = s_info[0];
  if (n == 0) return;
  const uint64_t cta_stride = 2ull * p.batch * 128;
  const uint32_t per_row = p.batch * 128;
  for (uint32_t e = threadIdx.x; e < n * per_row; e += nthreads) {
    const uint32_t k = e / per_row, rem = e - k * per_row, b = rem >> 7, rit = rem & 127;
    const uint32_t r = s_info[1 + 4 * k], first = s_info[2 + 4 * k], last = s_info[3 + 4 * k];
    const uint32_t row = r * 128 + rit;
    if (row >= p.rows) continue;
    const float* src = p.partials + static_cast<uint64_t>(b) * 128 + rit;
    float sum = 0.0f;
    // contributors in groups of 8: the loads of a group are independent, the sum is in order
    for (uint32_t i0 = first; i0 <= last; i0 += 8) {
      float v[8];
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j) {
        const uint32_t i = i0 + j;
        const uint64_t off = i * cta_stride + (i == first ? s_info[4 + 4 * k] * p.batch * 128 : 0u);
        v[j] = i <= last ? __ldcg(src + off) : 0.0f;
      }
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j)
        if (i0 + j <= last) {
          sum += v[j];
          // the partials region is zero between launches
          const uint64_t off = (i0 + j) * cta_stride + (i0 + j == first ? s_info[4 + 4 * k] * p.batch * 128 : 0u);
          __stcg(const_cast<float*>(src) + off, 0.0f);
        }
    }
    if (p.bias != nullptr)
      sum += p.bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(p.bias)[row])
                                     : static_cast<const float*>(p.bias)[row];
    put_y(p, b, row, sum);
  }
}

// Fused all-gather completion: after every CTA of the launch has stored its outputs (a
// system-scope fence orders the CTA's peer stores first), the last CTA adds 1 to this
// rank's counter in every rank's flag array with a system-scope release.
__device__ __forceinline__ void gather_signal(const GemvParams& p, uint32_t ctas) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atom_add_acq_rel_gpu(p.g_done, 1u) == ctas - 1) {
      *p.g_done = 0u;  // ready for the next launch
      for (uint32_t r = 0; r < p.g_world; ++r) red_add_release_sys(p.g_peer_flags[r] + p.g_rank, 1u);
    }
  }
}

// Tile columns a CTA needs: one range [a0, a1], plus [b0, b1] when its tiles wrap from
// the end of one tile row into the start of the next without covering every column.
struct ColRanges {
  uint32_t a0, a1, b0, b1;  // b1 < b0: no second range
  __device__ __forceinline__ uint32_t count() const { return (a1 - a0 + 1) + (b1 >= b0 ? b1 - b0 + 1 : 0); }
  __device__ __forceinline__ uint32_t col(uint32_t i) const { return i <= a1 - a0 ? a0 + i : b0 + (i - (a1 - a0 + 1)); }
};

__device__ __forceinline__ ColRanges needed_columns(uint32_t t0, uint32_t t_end, uint32_t C) {
  const uint32_t r0 = t0 / C, r1 = t_end / C, c0 = t0 - r0 * C, c1 = t_end - r1 * C;
  if (r0 == r1) return ColRanges{c0, c1, 1, 0};
  if (r1 == r0 + 1 && c1 + 1 < c0) return ColRanges{c0, C - 1, 0, c1};
  return ColRanges{0, C - 1, 1, 0};
}

// Activation fragments of the needed tile columns, built from raw x (FP16 for XL 1,
// FP32 for XL 2) by the CTA itself through prep_items, so they are bit-identical to a
// separately prepared buffer.  Each warp reads its items' activations straight from
// global memory, two items at a time, so their shuffle chains interleave.
// Resident activation slot of tile column c in a CTA whose first tile is in column
// c_first: (c - c_first) mod C.  The CTA walks its tiles in descending order, so it visits
// slots n-1, n-2, ..., 0 (mod C), and holds min(C, n) slots for n tiles.
__device__ __forceinline__ uint32_t resident_slot(uint32_t c, uint32_t c_first, uint32_t C) {
  return c >= c_first ? c - c_first : c + C - c_first;
}

// This lane's offsets in an int8 limb slot: its B fragment (N column g carries limb g/2
// of batch row g%2; at batch 1 the odd columns read entry 0, their accumulator columns
// are never stored) and the {L, K} pairs of its accumulator columns 2q and 2q+1.
struct XLaneI8 {
  uint32_t frag, cst;
  __device__ __forceinline__ XLaneI8(uint32_t batch, uint32_t lane) {
    const uint32_t g = lane >> 2, q = lane & 3;
    uint32_t entry = 0;
    if (g < 2 * kLimbs) entry = batch == 1 ? ((g & 1) ? 0u : g >> 1) : g;
    frag = entry * 128 + q * 32;
    cst = kLimbs * batch * 128 + q * 16;
  }
};

struct XFragI8 {
  uint32_t bf[4][2];  // [MMA m][b0, b1]
  float L[2], K[2];   // accumulator columns 2q, 2q+1
};

template <bool B1>
__device__ __forceinline__ void load_xfrag_i8(XFragI8& xf, const XLaneI8& xl, const uint8_t* slot) {
  const uint4 t0 = lds128(slot + xl.frag), t1 = lds128(slot + xl.frag + 16);
  xf.bf[0][0] = t0.x;
  xf.bf[0][1] = t0.y;
  xf.bf[1][0] = t0.z;
  xf.bf[1][1] = t0.w;
  xf.bf[2][0] = t1.x;
  xf.bf[2][1] = t1.y;
  xf.bf[3][0] = t1.z;
  xf.bf[3][1] = t1.w;
  if (B1) {
    const float2 c = lds_f2(slot + xl.cst);
    xf.L[0] = c.x;
    xf.K[0] = c.y;
    xf.L[1] = xf.K[1] = 0.0f;
  } else {
    const uint4 c = lds128(slot + xl.cst);
    xf.L[0] = __uint_as_float(c.x);
    xf.K[0] = __uint_as_float(c.y);
    xf.L[1] = __uint_as_float(c.z);
    xf.K[1] = __uint_as_float(c.w);
  }
}

// Integer tensor-core part of one tile: per stage 4 MMAs m16n8k32, MMA m fed by the
// code words ANDed with 0x03030303 << 2m (no shifts).  D independent accumulator chains
// (two for D == 1, the second starting from zero); every chain of a stage starts from
// the bits of 1.5·2^23.
template <int D, bool MX = false>
__device__ __forceinline__ void tile_mma_i8(const uint4 (&w)[D], const XFragI8& xf,
                                            uint32_t (&acc)[TileChains<D>::value][4], uint32_t live = ~0u) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t mask = 0x03030303u << (2 * m);
#pragma unroll
    for (int s = 0; s < D; ++s) {
      if (MX && !((live >> s) & 1u)) continue;  // warp-uniform: a stage the tile does not select
      const int c = D == 1 ? (m & 1) : s;
      const uint32_t a0 = w[s].x & mask, a1 = w[s].y & mask, a2 = w[s].z & mask, a3 = w[s].w & mask;
      if (D == 1 ? m < 2 : m == 0)
        mma_u8s8_seed(acc[c], a0, a1, a2, a3, xf.bf[m][0], xf.bf[m][1], (D == 1 && c == 1) ? 0u : kAccBiasBits);
      else
        mma_u8s8(acc[c], a0, a1, a2, a3, xf.bf[m][0], xf.bf[m][1]);
    }
  }
}

// y += σ·Σcode·Y·L per stage: one FMA turns the biased accumulator into the exact limb
// sum, one more applies the row's scale.  Each lane holds its own limb columns; the
// lane quad is summed when a tile row ends (quad_sum).
template <int D, bool B1, bool MX = false>
__device__ __forceinline__ void tile_epilogue_i8(const uint32_t (&sc)[D], const XFragI8& xf,
                                                 uint32_t (&acc)[TileChains<D>::value][4], float (&y)[1][4],
                                                 uint32_t live = ~0u) {
  if (D == 1) {
    acc[0][0] += acc[1][0];
    acc[0][2] += acc[1][2];
    if (!B1) {
      acc[0][1] += acc[1][1];
      acc[0][3] += acc[1][3];
    }
  }
#pragma unroll
  for (int s = 0; s < D; ++s) {
    if (MX && !((live >> s) & 1u)) continue;
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sc[s]);
    const float s_lo = __low2float(s2), s_hi = __high2float(s2);
    y[0][0] = fmaf(s_lo, fmaf(__uint_as_float(acc[s][0]), xf.L[0], xf.K[0]), y[0][0]);
    y[0][2] = fmaf(s_hi, fmaf(__uint_as_float(acc[s][2]), xf.L[0], xf.K[0]), y[0][2]);
    if (!B1) {
      y[0][1] = fmaf(s_lo, fmaf(__uint_as_float(acc[s][1]), xf.L[1], xf.K[1]), y[0][1]);
      y[0][3] = fmaf(s_hi, fmaf(__uint_as_float(acc[s][3]), xf.L[1], xf.K[1]), y[0][3]);
    }
  }
}

// Sum of the lane quad's limb columns; every lane of the quad ends with the same bits.
template <bool B1>
__device__ __forceinline__ void quad_sum(float (&y)[1][4]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (B1 && (e & 1)) continue;
    y[0][e] += __shfl_xor_sync(0xffffffffu, y[0][e], 1);
    y[0][e] += __shfl_xor_sync(0xffffffffu, y[0][e], 2);
  }
}

// ---- per-tile depth maps in the stream-K kernel ---------------------------------------
//
// Units are (tile, stage) pairs in tile order, Σ depth of them in all (plan[R]); CTA i of
// G takes [⌊iT/G⌋, ⌊(i+1)T/G⌋) as for a uniform prefix.  Each warp finds its CTA's range
// ends itself through L2 (no CTA barrier): the total and the rows holding the ends by a
// 32-way search of the plan, the tiles by a warp scan of those rows' depths.

// Largest r < R with plan[r] <= u (plan[0] = 0 <= u < plan[R]), with plan[r] and
// plan[r + 1]; every lane returns the same values.
__device__ __forceinline__ uint32_t plan_row_of(const uint32_t* plan, uint32_t R, uint64_t u, uint32_t lane,
                                                uint64_t& rb, uint64_t& re) {
  uint32_t lo = 0, hi = R;  // plan[lo] <= u < plan[hi]
  while (hi - lo > 1) {
    const uint32_t step = (hi - lo + 31) / 32;
    const uint32_t idx = lo + lane * step;
    const bool le = idx < hi && static_cast<uint64_t>(__ldg(plan + idx)) <= u;
    const uint32_t k = 31 - __clz(__ballot_sync(0xffffffffu, le));  // lane 0 always qualifies
    lo += k * step;
    hi = min(hi, lo + step);
  }
  rb = __ldg(plan + lo);
  re = __ldg(plan + lo + 1);
  return lo;
}

// Tile column c and stage s of the unit `off` units into tile row r (off < the row's units).
__device__ __forceinline__ void row_unit_tile(const GemvParams& p, uint32_t r, uint32_t off, uint32_t lane,
                                              uint32_t& c, uint32_t& s) {
  const uint8_t* row = p.depth + static_cast<uint64_t>(r) * p.C;
  uint32_t before = 0;
  for (uint32_t c0 = 0; c0 < p.C; c0 += 32) {
    const uint32_t d = c0 + lane < p.C ? clamp_depth(__ldg(row + c0 + lane), p.stage_count) : 0u;
    uint32_t incl = d;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= static_cast<uint32_t>(o)) incl += t;
    }
    const uint32_t m = __ballot_sync(0xffffffffu, before + incl > off);
    if (m != 0) {
      const uint32_t k = __ffs(m) - 1;
      c = c0 + k;
      s = off - before - __shfl_sync(0xffffffffu, incl - d, k);
      return;
    }
    before += __shfl_sync(0xffffffffu, incl, 31);
  }
  c = p.C - 1;  // not reached for a valid plan
  s = 0;
}

struct MixedRange {
  uint64_t total, u0, u1;
  uint64_t rb_first, re_last;  // first unit of the range's first row, end of its last row
  uint32_t ctas, t0, s0, t_end, s_end;
};

__device__ __forceinline__ MixedRange mixed_range(const GemvParams& p, uint32_t cta, uint32_t lane) {
  MixedRange m{};
  m.total = __ldg(p.plan + p.R);
  m.ctas = static_cast<uint32_t>(m.total < gridDim.x ? m.total : gridDim.x);
  if (cta >= m.ctas) return m;
  m.u0 = unit_start(cta, m.total, m.ctas);
  m.u1 = unit_start(cta + 1, m.total, m.ctas);
  uint64_t rb0, re0, rb1, re1;
  const uint32_t r0 = plan_row_of(p.plan, p.R, m.u0, lane, rb0, re0);
  const uint32_t r1 = plan_row_of(p.plan, p.R, m.u1 - 1, lane, rb1, re1);
  uint32_t c0, s0, c1, s1;
  row_unit_tile(p, r0, static_cast<uint32_t>(m.u0 - rb0), lane, c0, s0);
  row_unit_tile(p, r1, static_cast<uint32_t>(m.u1 - 1 - rb1), lane, c1, s1);
  m.rb_first = rb0;
  m.re_last = re1;
  m.t0 = r0 * p.C + c0;
  m.s0 = s0;
  m.t_end = r1 * p.C + c1;
  m.s_end = s1 + 1;
  return m;
}

// ---- int8-limb tile step from zero-started chains (bulk and lean stream-K kernels) ----

// D = A·B, m16n8k32 u8 x s8 -> s32, accumulator from zero.
__device__ __forceinline__ void mma_u8s8_z(uint32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0u));
}

// Integer tensor-core part of one tile: per stage 4 MMAs m16n8k32, MMA m fed by the code
// words ANDed with 0x03030303 << 2m.  D independent chains from zero (two for D == 1).
template <int D, bool MX>
__device__ __forceinline__ void bulk_tile_mma(const uint4 (&w)[D], const XFragI8& xf,
                                              uint32_t (&acc)[TileChains<D>::value][4], uint32_t live) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t mask = 0x03030303u << (2 * m);
#pragma unroll
    for (int s = 0; s < D; ++s) {
      if (MX && !((live >> s) & 1u)) continue;  // warp-uniform: a stage the tile does not select
      const int c = D == 1 ? (m & 1) : s;
      const uint32_t a0 = w[s].x & mask, a1 = w[s].y & mask, a2 = w[s].z & mask, a3 = w[s].w & mask;
      if (D == 1 ? m < 2 : m == 0)
        mma_u8s8_z(acc[c], a0, a1, a2, a3, xf.bf[m][0], xf.bf[m][1]);
      else
        mma_u8s8(acc[c], a0, a1, a2, a3, xf.bf[m][0], xf.bf[m][1]);
    }
  }
}

// y += σ·Σcode·Y·L per stage.  The integer sum S reads as the FP32 1.5·2^23 + S once the
// bits of 1.5·2^23 are added (|S| < 2^21), so one FMA with the slot's {L, K} gives the
// exact limb sum and one more applies the row's scale -- the arithmetic of the seeded
// chains of the register-ring kernels, bit for bit.
template <int D, bool B1, bool MX>
__device__ __forceinline__ void bulk_tile_epilogue(const uint32_t (&sc)[D], const XFragI8& xf,
                                                   uint32_t (&acc)[TileChains<D>::value][4], float (&y)[1][4],
                                                   uint32_t live) {
  if (D == 1) {
    acc[0][0] += acc[1][0];
    acc[0][2] += acc[1][2];
    if (!B1) {
      acc[0][1] += acc[1][1];
      acc[0][3] += acc[1][3];
    }
  }
#pragma unroll
  for (int s = 0; s < D; ++s) {
    if (MX && !((live >> s) & 1u)) continue;
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sc[s]);
    const float s_lo = __low2float(s2), s_hi = __high2float(s2);
    y[0][0] = fmaf(s_lo, fmaf(__uint_as_float(acc[s][0] + kAccBiasBits), xf.L[0], xf.K[0]), y[0][0]);
    y[0][2] = fmaf(s_hi, fmaf(__uint_as_float(acc[s][2] + kAccBiasBits), xf.L[0], xf.K[0]), y[0][2]);
    if (!B1) {
      y[0][1] = fmaf(s_lo, fmaf(__uint_as_float(acc[s][1] + kAccBiasBits), xf.L[1], xf.K[1]), y[0][1]);
      y[0][3] = fmaf(s_hi, fmaf(__uint_as_float(acc[s][3] + kAccBiasBits), xf.L[1], xf.K[1]), y[0][3]);
    }
  }
}

// Limb slots of the tile columns a CTA touches, built from raw x by WARPS warps.  Each
// lane loads four consecutive activations (one 8- or 16-byte load, no sector read twice),
// a per-warp 512-byte shared-memory area turns them into limb_item's column order, and the
// next item's load is in flight while the current one is transformed.  The loop is kept
// rolled: it runs once per launch from a cold instruction cache, where a compact body
// (one limb_item) costs less than unrolled ones.
template <int XL, uint32_t WARPS>
__device__ __forceinline__ void build_limb_slots(const GemvParams& p, uint8_t* xres, float* scratch,
                                                 const ColRanges& cr, uint32_t c_first, uint32_t warp, uint32_t lane) {
  using XT = typename std::conditional<XL == 1, __half, float>::type;
  const XT* x = static_cast<const XT*>(p.x_raw);
  const uint32_t items = cr.count() * p.batch;
  const uint32_t q = lane >> 3, m = (lane >> 1) & 3u, h = lane & 1u;
  const uint32_t col_lane = 32u * q + 16u * h + m;  // limb_item's columns: col_lane + 4j
  auto fetch = [&](uint32_t it, float (&v)[4], uint32_t& c, uint32_t& b) {
    const uint32_t ci = p.batch == 1 ? it : it >> 1;  // batch <= 2
    b = it - ci * p.batch;
    c = cr.col(ci);
    load_x4<XT>(x + static_cast<uint64_t>(b) * p.cols, c * 128 + 4 * lane, p.cols, p.x_vec != 0, v);
  };
  uint32_t it = warp;
  if (it >= items) return;
  float v[4];
  uint32_t c, b;
  fetch(it, v, c, b);
#pragma unroll 1
  for (; it < items; it += WARPS) {
    float vn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    uint32_t cn = 0, bn = 0;
    if (it + WARPS < items) fetch(it + WARPS, vn, cn, bn);
    *reinterpret_cast<float4*>(scratch + 4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
    __syncwarp();
    float u[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) u[jj] = scratch[col_lane + 4 * jj];
    __syncwarp();
    limb_item(u, xres + resident_slot(c, c_first, p.C) * p.xslot_bytes, b, p.batch, lane);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) v[jj] = vn[jj];
    c = cn;
    b = bn;
  }
}

// The same for a tile with a batch row whose limb slot is marked wide (K >= 0, see
// limb_item): such a row's K holds -K and its stage sums are multiplied by its wide factor
// (1.0 for the other row); NaN constants (a non-finite activation) give NaN.
template <int D, bool B1, bool MX>
__device__ __forceinline__ void bulk_tile_epilogue_wide(const uint32_t (&sc)[D], const XFragI8& xf,
                                                        uint32_t (&acc)[TileChains<D>::value][4], float (&y)[1][4],
                                                        uint32_t live, float f0, float f1) {
  if (D == 1) {
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[0][e] += acc[1][e];
  }
  // a wide row's K is stored negated (>= 0); NaN stays NaN
  const float k0 = xf.K[0] >= 0.0f ? -xf.K[0] : xf.K[0], k1 = xf.K[1] >= 0.0f ? -xf.K[1] : xf.K[1];
#pragma unroll
  for (int s = 0; s < D; ++s) {
    if (MX && !((live >> s) & 1u)) continue;
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sc[s]);
    const float s_lo = __low2float(s2), s_hi = __high2float(s2);
    y[0][0] = fmaf(s_lo * f0, fmaf(__uint_as_float(acc[s][0] + kAccBiasBits), xf.L[0], k0), y[0][0]);
    y[0][2] = fmaf(s_hi * f0, fmaf(__uint_as_float(acc[s][2] + kAccBiasBits), xf.L[0], k0), y[0][2]);
    if (!B1) {
      y[0][1] = fmaf(s_lo * f1, fmaf(__uint_as_float(acc[s][1] + kAccBiasBits), xf.L[1], k1), y[0][1]);
      y[0][3] = fmaf(s_hi * f1, fmaf(__uint_as_float(acc[s][3] + kAccBiasBits), xf.L[1], k1), y[0][3]);
    }
  }
}

// This lane's limb fragments and {L, K} from a slot at shared address `a` (XLaneI8 offsets).
template <bool B1>
__device__ __forceinline__ void load_limbs(XFragI8& xf, uint32_t frag_a, uint32_t cst_a) {
  const uint4 t0 = lds128a(frag_a), t1 = lds128a(frag_a + 16);
  xf.bf[0][0] = t0.x;
  xf.bf[0][1] = t0.y;
  xf.bf[1][0] = t0.z;
  xf.bf[1][1] = t0.w;
  xf.bf[2][0] = t1.x;
  xf.bf[2][1] = t1.y;
  xf.bf[3][0] = t1.z;
  xf.bf[3][1] = t1.w;
  if (B1) {
    const uint2 c = lds64a(cst_a);
    xf.L[0] = __uint_as_float(c.x);
    xf.K[0] = __uint_as_float(c.y);
    xf.L[1] = xf.K[1] = 0.0f;
  } else {
    const uint4 c = lds128a(cst_a);
    xf.L[0] = __uint_as_float(c.x);
    xf.K[0] = __uint_as_float(c.y);
    xf.L[1] = __uint_as_float(c.z);
    xf.K[1] = __uint_as_float(c.w);
  }
}

using GemvKernel = void (*)(GemvParams);

// Launch shape of the bulk-copy GEMV (hqb_bulk.cu).
struct BulkPlan {
  uint32_t grid, per_sm, slots, chunk_tiles, chunk_bytes, res_slots, smem;
};
BulkPlan bulk_plan(uint64_t tiles, uint32_t depth, bool mixed, uint32_t C, uint32_t xslot, int sms);
uint32_t bulk_smem_max();
cudaError_t launch_gemv_bulk(GemvParams p, const BulkPlan& b, uint32_t depth, uint32_t xl, bool mx, bool pdl,
                             cudaStream_t st);
cudaError_t launch_prep_limbs(const void* x, int x_dtype, uint64_t cols, uint32_t batch, void* xfrag, bool pdl,
                              cudaStream_t st);

}  // namespace hqb
