// Plane-layout kernels of the progressive int2 GEMV for sm_100a.
//
//   repack_kernel        reference row-major stage -> plane records (one per tile)
//   prep_x_kernel        activations -> per-tile FP16 tensor-core B fragments + correction sums
//   gemv_uniform_kernel  stream-K GEMV with a per-warp register ring (uniform prefix; the
//                        int8 form runs lean_body); split tile rows finished in-kernel
//   gemv_unit_kernel     stream-K GEMV for a depth map on the int8 form, one (tile, stage)
//                        unit per ring slot
//   gemv_grouped_kernel  independent GEMVs in one launch (lean_body per problem)
//   gemv_rows_kernel     row-block GEMV for small layers (no tile row split between CTAs)
//   gemv_stream_kernel   depth maps where the int8 form does not apply
//   gemv_kernel          warp-specialised, bulk-copy pipelined GEMV (tensor-core or CUDA-core
//                        consumer) for wide activations and comparisons, with fixup_kernel
//   gemv_tc_kernel       tcgen05 (UMMA, TMEM accumulators) comparison GEMV
//   decode_kernel        planes -> dense FP32 weights, bit-identical to DequantizePrefix
//   depth_plan_kernel    per-tile depth map -> row-cost prefix sums (the mixed-depth schedule)
//   fill_kernel          prefix 0: bias or exact zeros
//
// Plane record of one (tile, stage), HQB_TILE_RECORD_BYTES = 8 x 544:
//   row block rb (tile rows 16rb..16rb+15) at rb*544:
//     [0, 512)   32 slots of 16 B, slot t = 4g+q holds four 32-bit code words
//                  w0 = row 16rb+g,   columns 32q..32q+15     (2 bits/code, LSB first,
//                                                              stored as code + 2)
//                  w1 = row 16rb+g+8, columns 32q..32q+15
//                  w2 = row 16rb+g,   columns 32q+16..32q+31
//                  w3 = row 16rb+g+8, columns 32q+16..32q+31
//                so lane t of a warp gets exactly its m16n8k16 A-fragment codes with
//                one 16-byte shared-memory load;
//     [512, 544) 8 pairs {scale(row 16rb+g), scale(row 16rb+g+8)} as raw FP16 bits.
//
// Tensor-core decode: code pair j of each 16-bit half (positions 0..3 of w, 4..7 of
// w >> 8) becomes the FP16 subnormal (code+2)·4^(j%4)·2^-24 with one AND (the plane
// stores code + 2).  The B operand holds x·2^-e·4^-(j%4) (per-tile exponent e), so every
// product is (code+2)·x·2^(-24-e) and the FP32 accumulator of one tile-stage is
// 2^(-24-e)·Σ(code+2)·x.  The epilogue applies f = 2^(24+e), subtracts the
// row-independent 2·Σx term and multiplies by the row's FP16 scale.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>
#include <type_traits>

#include "harpq_b200.h"
#include "hqb_device.cuh"
#include "hqb_internal.h"
#include "hqb_schedule.h"
#include "hqb_gemv_common.cuh"

namespace hqb {


// --------------------------------------------------------------------------------------
// repack

__global__ void __launch_bounds__(256) repack_kernel(const uint8_t* __restrict__ codes,
                                                     const uint16_t* __restrict__ scales,
                                                     uint8_t* __restrict__ plane,
                                                     uint64_t row_bytes, uint32_t rows,
                                                     uint32_t cols, uint32_t C, int* flags,
                                                     int aligned4) {
  const uint32_t tile = blockIdx.x;
  const uint32_t r = tile / C, c = tile % C;
  const uint32_t rb = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  uint32_t words[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t row = r * 128 + rb * 16 + g + 8 * (i & 1);
    const uint32_t col0 = c * 128 + 32 * q + 16 * (i >> 1);
    uint32_t w = 0;
    if (row < rows && col0 < cols) {
      const uint8_t* src = codes + static_cast<uint64_t>(row) * row_bytes + c * 32 + 8 * q + 4 * (i >> 1);
      w = aligned4 ? *reinterpret_cast<const uint32_t*>(src)
                   : (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) |
                         ((uint32_t)src[3] << 24);
      const uint32_t valid = cols - col0;
      if (valid < 16) w &= (1u << (2 * valid)) - 1u;  // padded columns get code 0
    }
    // Store every 2-bit field as (code + 2) in [0, 3] (two's-complement raw XOR 0b10):
    // the tensor-core decode is then a single AND per register.
    words[i] = w ^ 0xAAAAAAAAu;
  }
  uint8_t* rec = plane + static_cast<uint64_t>(tile) * kRecordBytes + rb * kRowBlockBytes;
  *reinterpret_cast<uint4*>(rec + lane * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  if (lane < 8) {
    const uint64_t base = static_cast<uint64_t>(tile) * 128 + rb * 16 + lane;
    const uint32_t s0 = scales[base], s1 = scales[base + 8];
    int bad = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t s = k ? s1 : s0;
      if (((s >> 10) & 0x1F) == 0x1F || ((s & 0x8000u) && (s & 0x7FFFu))) bad = 1;
    }
    if (bad && flags != nullptr) atomicOr(flags, HQB_DEVERR_SCALE);
    *reinterpret_cast<uint32_t*>(rec + 512 + lane * 4) = s0 | (s1 << 16);
  }
}


// x [batch][cols] -> one fragment slot per 128-column tile; one warp per (tile column,
// batch row) item, four items per block.
template <int XL, typename XT>
__global__ void __launch_bounds__(128) prep_x_kernel(const XT* __restrict__ x, uint32_t cols, uint32_t batch,
                                                     uint32_t C, uint8_t* __restrict__ xfrag, uint32_t xslot,
                                                     uint32_t vec) {
  const uint32_t item = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= C * batch) return;  // the whole warp leaves together
  const uint32_t c = item / batch;
  float v[1][4];
  const bool ok[1] = {true};
  uint8_t* const slot[1] = {xfrag + static_cast<uint64_t>(c) * xslot};
  const uint32_t b[1] = {item - c * batch};
  load_x4<XT>(x + static_cast<uint64_t>(b[0]) * cols, c * 128 + 4 * lane, cols, vec != 0, v[0]);
  prep_items<XL, 1>(v, ok, slot, b, batch, lane);
}

// --------------------------------------------------------------------------------------
// GEMV
//
// Warp roles per CTA: warp 8 lane 0 is the producer; warps 0..7 are consumers, warp w
// owning rows 16w..16w+15 of every tile.  The CTA's unit range is walked as "runs":
// stages [s0, s1) of one tile.  One ring slot carries one run:
//     [16-byte header][activation fragments of the tile][record s0]...[record s1-1]
// The producer alone walks the schedule (uniform prefix or depth map), writes the
// header and issues the bulk copies; consumers only follow headers.

constexpr uint32_t kHdrBytes = 16;
constexpr uint32_t kFlagFlush = 1;  // this run ends the CTA's part of its tile row
constexpr uint32_t kFlagLast = 2;   // last run of the CTA
constexpr uint32_t kFlagError = 4;  // schedule error: consumers stop

struct RunCursor {
  uint32_t r, c, s, left;

  __device__ bool init(uint64_t u, uint32_t n, const GemvParams& p) {
    left = n;
    if (p.plan == nullptr) {
      const uint64_t per_row = static_cast<uint64_t>(p.C) * p.prefix;
      r = static_cast<uint32_t>(u / per_row);
      const uint64_t rem = u - static_cast<uint64_t>(r) * per_row;
      c = static_cast<uint32_t>(rem / p.prefix);
      s = static_cast<uint32_t>(rem - static_cast<uint64_t>(c) * p.prefix);
      return true;
    }
    r = row_of_unit(u, p.plan, p.R, 0);
    uint64_t off = u - p.plan[r];
    for (c = 0; c < p.C; ++c) {
      const uint32_t d = clamp_depth(p.depth[static_cast<uint64_t>(r) * p.C + c], p.stage_count);
      if (off < d) {
        s = static_cast<uint32_t>(off);
        return true;
      }
      off -= d;
    }
    return false;  // plan and depth map disagree
  }

  // Next run; false when the schedule walks past the last tile row (inconsistent plan).
  __device__ bool next(const GemvParams& p, uint32_t& rr, uint32_t& cc, uint32_t& s0, uint32_t& s1,
                       uint32_t& flags) {
    if (r >= p.R) return false;
    const uint32_t d = p.plan == nullptr ? p.prefix : clamp_depth(p.depth[static_cast<uint64_t>(r) * p.C + c], p.stage_count);
    rr = r;
    cc = c;
    s0 = s;
    s1 = min(d, s + left);
    left -= s1 - s0;
    s = 0;
    flags = 0;
    if (++c == p.C) {
      c = 0;
      ++r;
      flags |= kFlagFlush;
    }
    if (left == 0) flags |= kFlagFlush | kFlagLast;
    return true;
  }
};

struct Ring {
  uint8_t* base;
  uint8_t* xres;  // resident activation fragments (x_resident)
  uint64_t* full;
  uint64_t* empty;
  uint64_t* xbar;
  uint32_t slots, stride;
};

// The producer warp: lane 0 walks the schedule, writes the slot header and arms the
// slot's barrier with the byte count; then lanes 0..len-1 issue one stage record each
// and lane 31 the tile's activation fragments, so a slot costs one warp step rather
// than a serial chain of copies on one thread.
__device__ void gemv_producer(const GemvParams& p, const Ring& ring, uint64_t u0, uint32_t n, uint32_t lane) {
  const uint64_t stream_policy = policy_evict_first();
  const uint64_t keep_policy = policy_evict_last();
  RunCursor rc;
  bool ok = true;
  if (lane == 0) ok = rc.init(u0, n, p);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) {
    if (lane == 0) {
      atomicOr(p.error, HQB_DEVERR_DEPTH);
      uint32_t* hdr = reinterpret_cast<uint32_t*>(ring.base);
      hdr[0] = hdr[1] = 0;
      hdr[2] = (kFlagLast | kFlagError) << 16;
      mbar_arrive(&ring.full[0]);  // a header-only phase tells the consumers to stop
    }
    return;
  }
  // With programmatic dependent launch the activation fragments may still be written
  // by the preceding kernel: weight records go first, activations after the wait.
  const bool defer_x = p.pdl != 0;
  bool x_pending = defer_x;  // prologue activations not yet issued
  if (p.x_resident && lane == 0) {
    mbar_expect_tx(ring.xbar, static_cast<uint32_t>(p.C) * p.xslot_bytes);
    if (!defer_x) bulk_load(ring.xres, p.xfrag, static_cast<uint32_t>(p.C) * p.xslot_bytes, ring.xbar, keep_policy);
  }
  __syncwarp();
  uint32_t k = 0;
  bool last = false;
  while (!last) {
    const uint32_t i = k % ring.slots;
    uint8_t* slot = ring.base + i * ring.stride;
    if (k == ring.slots && x_pending) {
      x_pending = false;
      griddep_wait();
      if (p.x_resident) {
        if (lane == 0)
          bulk_load(ring.xres, p.xfrag, static_cast<uint32_t>(p.C) * p.xslot_bytes, ring.xbar, keep_policy);
      } else
      for (uint32_t j = lane; j < ring.slots; j += 32) {  // activations of the prologue slots
        uint8_t* sj = ring.base + j * ring.stride;
        const uint32_t* hj = reinterpret_cast<const uint32_t*>(sj);
        if ((hj[2] >> 16) & kFlagError) continue;
        bulk_load(sj + kHdrBytes, p.xfrag + static_cast<uint64_t>(hj[1]) * p.xslot_bytes, p.xslot_bytes,
                  &ring.full[j], keep_policy);
      }
    }
    uint32_t r = 0, c = 0, s0 = 0, s1 = 0, flags = 0;
    bool waited = true, valid = true;
    if (lane == 0) {
      if (k >= ring.slots) waited = mbar_wait(&ring.empty[i], ((k / ring.slots) - 1) & 1, p.error);
      if (waited) {
        valid = rc.next(p, r, c, s0, s1, flags);
        uint32_t* hdr = reinterpret_cast<uint32_t*>(slot);
        if (!valid) {
          atomicOr(p.error, HQB_DEVERR_DEPTH);
          flags = kFlagLast | kFlagError;
          s0 = s1 = 0;
        }
        hdr[0] = r;
        hdr[1] = c;
        hdr[2] = (s1 - s0) | (flags << 16);
        mbar_expect_tx(&ring.full[i], valid ? p.slot_x_bytes + (s1 - s0) * kRecordBytes : 0);
      }
    }
    waited = __shfl_sync(0xffffffffu, waited, 0);
    if (!waited) break;
    r = __shfl_sync(0xffffffffu, r, 0);
    c = __shfl_sync(0xffffffffu, c, 0);
    s0 = __shfl_sync(0xffffffffu, s0, 0);
    s1 = __shfl_sync(0xffffffffu, s1, 0);
    flags = __shfl_sync(0xffffffffu, flags, 0);
    valid = (flags & kFlagError) == 0;
    last = (flags & kFlagLast) != 0;
    __syncwarp();  // the barrier is armed before any copy can complete on it
    if (valid) {
      if (lane < s1 - s0)
        bulk_load(slot + kHdrBytes + p.slot_x_bytes + lane * kRecordBytes,
                  p.planes[s0 + lane] + (static_cast<uint64_t>(r) * p.C + c) * kRecordBytes, kRecordBytes,
                  &ring.full[i], stream_policy);
      if (lane == 31 && !x_pending && !p.x_resident)
        bulk_load(slot + kHdrBytes, p.xfrag + static_cast<uint64_t>(c) * p.xslot_bytes, p.xslot_bytes,
                  &ring.full[i], keep_policy);
    }
    ++k;
  }
  if (x_pending) {  // schedules of at most ring.slots runs end before the wait above
    x_pending = false;
    griddep_wait();
    if (p.x_resident) {
      if (lane == 0)
        bulk_load(ring.xres, p.xfrag, static_cast<uint32_t>(p.C) * p.xslot_bytes, ring.xbar, keep_policy);
    } else
    for (uint32_t j = lane; j < k; j += 32) {
      uint8_t* sj = ring.base + j * ring.stride;
      const uint32_t* hj = reinterpret_cast<const uint32_t*>(sj);
      if ((hj[2] >> 16) & kFlagError) continue;
      bulk_load(sj + kHdrBytes, p.xfrag + static_cast<uint64_t>(hj[1]) * p.xslot_bytes, p.xslot_bytes, &ring.full[j],
                keep_policy);
    }
  }
  // Every bulk copy this CTA issued must land before the CTA may exit, whatever path
  // led here (consumers may have left early on an error).
  if (lane == 0) {
    for (uint32_t j = k > ring.slots ? k - ring.slots : 0; j < k; ++j)
      mbar_wait(&ring.full[j % ring.slots], (j / ring.slots) & 1, p.error);
    if (p.x_resident) mbar_wait(ring.xbar, 0, p.error);
  }
}


// Activation fragments of one tile for this lane (batch rows g and g+8).
template <int NB, int XL>
struct XFrag {
  uint32_t bf[NB][XL][8][2];
  float f[NB][2], gsum[NB][2];

  __device__ __forceinline__ void load(const GemvParams& p, const uint8_t* slot, uint32_t lane) {
    const uint32_t g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const uint32_t b = g + 8 * nb;
#pragma unroll
      for (int l = 0; l < XL; ++l) {
        if (b < p.batch) {
          const uint8_t* src = slot + l * p.batch * 256 + (b * 4 + q) * 64;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const uint4 t = lds128(src + 16 * v);
            bf[nb][l][2 * v][0] = t.x;
            bf[nb][l][2 * v][1] = t.y;
            bf[nb][l][2 * v + 1][0] = t.z;
            bf[nb][l][2 * v + 1][1] = t.w;
          }
        } else {
#pragma unroll
          for (int m = 0; m < 8; ++m) bf[nb][l][m][0] = bf[nb][l][m][1] = 0u;
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t bb = 2 * q + j + 8 * nb;
        float2 fg = make_float2(0.0f, 0.0f);
        if (bb < p.batch) fg = lds_f2(slot + p.batch * 256 * XL + bb * 8);
        f[nb][j] = fg.x;
        gsum[nb][j] = fg.y;
      }
    }
  }
};

// Code pair m (position m of each 16-bit half) as two FP16 subnormals (code+2)·4^(m%4)·2^-24:
// the plane stores code+2, so one AND extracts both.
__device__ __forceinline__ uint32_t int2_pair(uint32_t w, uint32_t w_hi, int m) {
  return ((m < 4) ? w : w_hi) & (0x00030003u << (2 * (m & 3)));
}

// LEN stages of one tile through the tensor cores: LEN independent accumulator chains.
template <int NB, int XL, int LEN>
__device__ __forceinline__ void mma_run(const XFrag<NB, XL>& xf, const uint4 (&w)[HQB_MAX_STAGES],
                                        const uint32_t (&sc)[HQB_MAX_STAGES], uint32_t shift_mul, float (&y)[NB][4]) {
  uint32_t hi[LEN][4];
#pragma unroll
  for (int j = 0; j < LEN; ++j) {
    // w >> 8 as a high multiply: runs on the FMA pipe and leaves the ALU pipe to the decode
    hi[j][0] = __umulhi(w[j].x, shift_mul);
    hi[j][1] = __umulhi(w[j].y, shift_mul);
    hi[j][2] = __umulhi(w[j].z, shift_mul);
    hi[j][3] = __umulhi(w[j].w, shift_mul);
  }
  float acc[LEN][NB][4];
#pragma unroll
  for (int j = 0; j < LEN; ++j)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][nb][e] = 0.0f;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
#pragma unroll
    for (int j = 0; j < LEN; ++j) {
      const uint32_t a0 = int2_pair(w[j].x, hi[j][0], m), a1 = int2_pair(w[j].y, hi[j][1], m);
      const uint32_t a2 = int2_pair(w[j].z, hi[j][2], m), a3 = int2_pair(w[j].w, hi[j][3], m);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int l = 0; l < XL; ++l) mma_f16(acc[j][nb], a0, a1, a2, a3, xf.bf[nb][l][m][0], xf.bf[nb][l][m][1]);
    }
  }
#pragma unroll
  for (int j = 0; j < LEN; ++j) {
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sc[j]);
    const float s_lo = __low2float(s2), s_hi = __high2float(s2);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      y[nb][0] = fmaf(s_lo, fmaf(acc[j][nb][0], xf.f[nb][0], -xf.gsum[nb][0]), y[nb][0]);
      y[nb][1] = fmaf(s_lo, fmaf(acc[j][nb][1], xf.f[nb][1], -xf.gsum[nb][1]), y[nb][1]);
      y[nb][2] = fmaf(s_hi, fmaf(acc[j][nb][2], xf.f[nb][0], -xf.gsum[nb][0]), y[nb][2]);
      y[nb][3] = fmaf(s_hi, fmaf(acc[j][nb][3], xf.f[nb][1], -xf.gsum[nb][1]), y[nb][3]);
    }
  }
}

// CUDA-core comparison consumer: each code decoded to FP32 with an exponent trick and
// one FFMA per code and batch row; partial column sums per lane are reduced across the
// lane quad when a tile row is finished.  Batch <= 8, FP16 activations.
__device__ __forceinline__ void simt_unit(const GemvParams& p, const uint8_t* xslot, uint32_t lane, const uint4 w,
                                          uint32_t sc, float (&part)[2][8]) {
  const uint32_t q = lane & 3;
  const __half2 s2 = *reinterpret_cast<const __half2*>(&sc);
  const float s_lo = __low2float(s2), s_hi = __high2float(s2);
#pragma unroll
  for (uint32_t b = 0; b < 8; ++b) {
    if (b >= p.batch) break;
    const float xsc = lds_f2(xslot + p.batch * 256 + b * 8).x * 0x1p-24f;  // 2^e of the tile
    const uint8_t* src = xslot + (b * 4 + q) * 64;
    uint32_t hx[16];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 t = lds128(src + 16 * v);
      hx[4 * v] = t.x;
      hx[4 * v + 1] = t.y;
      hx[4 * v + 2] = t.z;
      hx[4 * v + 3] = t.w;
    }
    float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int m = i & 7, which = i >> 3;
      const int idx = m * 4 + which;  // half index inside (b, q)
      const uint32_t hb = (idx & 1) ? (hx[idx >> 1] >> 16) : (hx[idx >> 1] & 0xFFFFu);
      const float xv = half_bits_to_float(hb) * static_cast<float>(1 << (2 * (m & 3)));
      const uint32_t wg = i < 16 ? w.x : w.z, wh = i < 16 ? w.y : w.w;
      const int sh = 2 * (i & 15);
      const float cg = __uint_as_float(0x4B000000u | ((wg >> sh) & 3u)) - 8388610.0f;
      const float ch = __uint_as_float(0x4B000000u | ((wh >> sh) & 3u)) - 8388610.0f;
      d0 = fmaf(cg, xv, d0);
      d1 = fmaf(ch, xv, d1);
    }
    part[0][b] = fmaf(s_lo * xsc, d0, part[0][b]);
    part[1][b] = fmaf(s_hi * xsc, d1, part[1][b]);
  }
}

__device__ __forceinline__ void simt_finish(float (&part)[2][8], float (&y)[1][4], uint32_t lane) {
  const uint32_t q = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      float v = part[h][b];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      part[h][b] = v;
    }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
    for (int b = 0; b < 8; ++b)
      if (static_cast<uint32_t>(b) == 2 * q + j) {
        v0 = part[0][b];
        v1 = part[1][b];
      }
    y[0][j] = v0;
    y[0][2 + j] = v1;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int b = 0; b < 8; ++b) part[h][b] = 0.0f;
}

template <int NB, int XL, bool SIMT>
__global__ void __launch_bounds__(kGemvThreads, (NB == 1 && XL == 1 && !SIMT) ? 2 : 1)
    gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint64_t total = p.plan != nullptr ? static_cast<uint64_t>(p.plan[p.R]) : p.total;
  // Mixed depth launches the full grid (the unit count lives on the device); both
  // modes partition over min(grid, units) CTAs so equal unit counts split equally.
  const uint32_t ctas = static_cast<uint32_t>(total < gridDim.x ? total : gridDim.x), cta = blockIdx.x;
  griddep_launch_dependents();  // the split-row fix-up may be scheduled; it waits for this grid
  if (cta >= ctas) return;
  const uint64_t u0 = unit_start(cta, total, ctas), u1 = unit_start(cta + 1, total, ctas);
  const uint32_t n = static_cast<uint32_t>(u1 - u0);

  Ring ring;
  ring.base = smem;
  ring.slots = p.ring_slots;
  ring.stride = p.slot_stride;
  ring.xres = smem + ring.slots * ring.stride;
  ring.full = reinterpret_cast<uint64_t*>(ring.xres + (p.x_resident ? p.C * p.xslot_bytes : 0));
  ring.empty = ring.full + ring.slots;
  ring.xbar = ring.empty + ring.slots;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < ring.slots; ++i) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], kConsumerWarps * 32);
    }
    mbar_init(ring.xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    gemv_producer(p, ring, u0, n, lane);
    return;
  }

  const uint32_t g = lane >> 2, q = lane & 3, rit0 = warp * 16 + g;
  const uint64_t per_row = static_cast<uint64_t>(p.C) * p.prefix;
  const uint32_t first_row = row_of_unit(u0, p.plan, p.R, per_row);
  float y[NB][4];
  float part[2][8];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) y[nb][e] = 0.0f;
  if constexpr (SIMT) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int b = 0; b < 8; ++b) part[h][b] = 0.0f;
  }
  griddep_wait();
  if (p.x_resident && !mbar_wait(ring.xbar, 0, p.error)) return;
  for (uint32_t k = 0;; ++k) {
    const uint32_t i = k % ring.slots;
    if (!mbar_wait(&ring.full[i], (k / ring.slots) & 1, p.error)) return;
    const uint8_t* slot = ring.base + i * ring.stride;
    const uint4 hdr = lds128(slot);
    const uint32_t len = hdr.z & 0xFFFFu, flags = hdr.z >> 16;
    if (flags & kFlagError) {
      mbar_arrive(&ring.empty[i]);
      return;
    }
    const uint8_t* xs = p.x_resident ? ring.xres + hdr.y * p.xslot_bytes : slot + kHdrBytes;
    const uint8_t* rec = slot + kHdrBytes + p.slot_x_bytes + warp * kRowBlockBytes;
    uint4 w[HQB_MAX_STAGES];
    uint32_t sc[HQB_MAX_STAGES];
#pragma unroll
    for (uint32_t j = 0; j < HQB_MAX_STAGES; ++j) {
      if (j < len) {
        w[j] = lds128(rec + j * kRecordBytes + lane * 16);
        sc[j] = lds32(rec + j * kRecordBytes + 512 + g * 4);
      }
    }
    if constexpr (SIMT) {
#pragma unroll
      for (uint32_t j = 0; j < HQB_MAX_STAGES; ++j)
        if (j < len) simt_unit(p, xs, lane, w[j], sc[j], part);
      mbar_arrive(&ring.empty[i]);
    } else {
      XFrag<NB, XL> xf;
      xf.load(p, xs, lane);
      mbar_arrive(&ring.empty[i]);  // every lane has its data in registers
      switch (len) {
        case 1: mma_run<NB, XL, 1>(xf, w, sc, p.shift_mul, y); break;
        case 2: mma_run<NB, XL, 2>(xf, w, sc, p.shift_mul, y); break;
        case 3: mma_run<NB, XL, 3>(xf, w, sc, p.shift_mul, y); break;
        default: mma_run<NB, XL, 4>(xf, w, sc, p.shift_mul, y); break;
      }
    }
    if (flags & kFlagFlush) {
      if constexpr (SIMT) simt_finish(part, reinterpret_cast<float(&)[1][4]>(y), lane);
      const uint32_t r = hdr.x;
      const RowSplit rs = row_split(p, r, total, ctas);
      if (rs.first == rs.last) {
        store_out<NB>(p, y, r * 128 + rit0, q);  // the whole tile row is this CTA's
      } else {
        // A split row: plain stores of this CTA's part; fixup_kernel adds the parts in
        // CTA order once the whole grid has finished (no fence or atomic here).
        publish_partial<NB>(p, cta, r == first_row ? 0 : 1, y, rit0, q);
      }
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) y[nb][e] = 0.0f;
    }
    if (flags & kFlagLast) break;
  }
}

// --------------------------------------------------------------------------------------
// Streaming GEMV (the batch <= 16 path whenever the activation fragments of a whole
// row fit in shared memory).  No producer warp and no ring: warp w owns rows
// 16w..16w+15 of every tile in the CTA's unit range and loads its own 544-byte
// row-block of each tile-stage straight into registers, kPrefetch units ahead, with
// 16-byte non-caching global loads.  The CTA's activation fragments are staged in
// shared memory once.  Partition, row flush and split-row fix-up are the ring kernel's.


struct UnitCursor {
  uint32_t r, c, s, d;

  __device__ bool init(uint64_t u, const GemvParams& p) {
    if (p.plan == nullptr) {
      const uint64_t per_row = static_cast<uint64_t>(p.C) * p.prefix;
      r = static_cast<uint32_t>(u / per_row);
      const uint64_t rem = u - static_cast<uint64_t>(r) * per_row;
      c = static_cast<uint32_t>(rem / p.prefix);
      s = static_cast<uint32_t>(rem - static_cast<uint64_t>(c) * p.prefix);
      d = p.prefix;
      return true;
    }
    r = row_of_unit(u, p.plan, p.R, 0);
    uint64_t off = u - p.plan[r];
    for (c = 0; c < p.C; ++c) {
      d = clamp_depth(p.depth[static_cast<uint64_t>(r) * p.C + c], p.stage_count);
      if (off < d) {
        s = static_cast<uint32_t>(off);
        return true;
      }
      off -= d;
    }
    return false;
  }

  __device__ __forceinline__ void advance(const GemvParams& p) {
    if (++s < d) return;
    s = 0;
    if (++c == p.C) {
      c = 0;
      ++r;
    }
    if (p.plan != nullptr && r < p.R) d = clamp_depth(p.depth[static_cast<uint64_t>(r) * p.C + c], p.stage_count);
  }
};

// This lane's 16 code bytes and scale pair of one tile-stage (read once: no L1 allocation).
__device__ __forceinline__ void load_unit(const GemvParams& p, const UnitCursor& u, uint32_t warp, uint32_t lane,
                                          uint4& w, uint32_t& sc) {
  const uint8_t* rec =
      p.planes[u.s] + (static_cast<uint64_t>(u.r) * p.C + u.c) * kRecordBytes + warp * kRowBlockBytes;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
               : "l"(rec + lane * 16));
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(sc) : "l"(rec + 512 + (lane >> 2) * 4));
}

template <int NB, int XL>
__device__ __forceinline__ void mma_unit(const XFrag<NB, XL>& xf, const uint4 w, uint32_t sc, uint32_t shift_mul,
                                         float (&y)[NB][4]) {
  const uint32_t h0 = __umulhi(w.x, shift_mul), h1 = __umulhi(w.y, shift_mul);
  const uint32_t h2 = __umulhi(w.z, shift_mul), h3 = __umulhi(w.w, shift_mul);
  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nb][e] = 0.0f;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const uint32_t a0 = int2_pair(w.x, h0, m), a1 = int2_pair(w.y, h1, m);
    const uint32_t a2 = int2_pair(w.z, h2, m), a3 = int2_pair(w.w, h3, m);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int l = 0; l < XL; ++l) mma_f16(acc[nb], a0, a1, a2, a3, xf.bf[nb][l][m][0], xf.bf[nb][l][m][1]);
  }
  const __half2 s2 = *reinterpret_cast<const __half2*>(&sc);
  const float s_lo = __low2float(s2), s_hi = __high2float(s2);
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    y[nb][0] = fmaf(s_lo, fmaf(acc[nb][0], xf.f[nb][0], -xf.gsum[nb][0]), y[nb][0]);
    y[nb][1] = fmaf(s_lo, fmaf(acc[nb][1], xf.f[nb][1], -xf.gsum[nb][1]), y[nb][1]);
    y[nb][2] = fmaf(s_hi, fmaf(acc[nb][2], xf.f[nb][0], -xf.gsum[nb][0]), y[nb][2]);
    y[nb][3] = fmaf(s_hi, fmaf(acc[nb][3], xf.f[nb][1], -xf.gsum[nb][1]), y[nb][3]);
  }
}

template <int NB, int XL>
__global__ void __launch_bounds__(kStreamThreads, (NB == 1 && XL == 1) ? 2 : 1)
    gemv_stream_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) uint8_t xres[];  // activation fragments, indexed by tile column
  const uint64_t total = p.plan != nullptr ? static_cast<uint64_t>(p.plan[p.R]) : p.total;
  const uint32_t ctas = static_cast<uint32_t>(total < gridDim.x ? total : gridDim.x), cta = blockIdx.x;
  griddep_launch_dependents();  // the split-row fix-up may be scheduled; it waits for this grid
  if (cta >= ctas) return;
  const uint64_t u0 = unit_start(cta, total, ctas), u1 = unit_start(cta + 1, total, ctas);
  const uint32_t n = static_cast<uint32_t>(u1 - u0);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const uint32_t rit0 = warp * 16 + g;

  UnitCursor fetch, cons, lastu;
  if (!fetch.init(u0, p) || !lastu.init(u1 - 1, p)) {
    if (threadIdx.x == 0) atomicOr(p.error, HQB_DEVERR_DEPTH);
    return;
  }
  cons = fetch;
  // Weight records do not depend on the preceding kernel: start them before the wait.
  uint4 w[kPrefetch];
  uint32_t sc[kPrefetch];
#pragma unroll
  for (int j = 0; j < kPrefetch; ++j) {
    if (static_cast<uint32_t>(j) < n) {
      load_unit(p, fetch, warp, lane, w[j], sc[j]);
      fetch.advance(p);
    }
  }
  griddep_wait();
  // Activation fragments of the tile columns this CTA touches (all of them when its
  // range crosses a tile row).
  {
    const uint32_t c_lo = cons.r == lastu.r ? cons.c : 0, c_hi = cons.r == lastu.r ? lastu.c : p.C - 1;
    const uint4* src = reinterpret_cast<const uint4*>(p.xfrag + static_cast<uint64_t>(c_lo) * p.xslot_bytes);
    uint4* dst = reinterpret_cast<uint4*>(xres + c_lo * p.xslot_bytes);
    const uint32_t chunks = (c_hi - c_lo + 1) * p.xslot_bytes / 16;
    for (uint32_t t = threadIdx.x; t < chunks; t += kStreamThreads) dst[t] = __ldcg(src + t);
  }
  __syncthreads();

  const uint64_t per_row = static_cast<uint64_t>(p.C) * p.prefix;
  const uint32_t first_row = row_of_unit(u0, p.plan, p.R, per_row);
  float y[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) y[nb][e] = 0.0f;
  XFrag<NB, XL> xf;
  uint32_t x_col = 0xFFFFFFFFu;
  for (uint32_t i = 0; i < n; i += kPrefetch) {
#pragma unroll
    for (int j = 0; j < kPrefetch; ++j) {
      if (i + j >= n) break;
      if (cons.c != x_col) {
        xf.load(p, xres + cons.c * p.xslot_bytes, lane);
        x_col = cons.c;
      }
      mma_unit<NB, XL>(xf, w[j], sc[j], p.shift_mul, y);
      if (i + j + kPrefetch < n) {
        load_unit(p, fetch, warp, lane, w[j], sc[j]);
        fetch.advance(p);
      }
      const uint32_t r = cons.r;
      cons.advance(p);
      if (i + j + 1 == n || cons.r != r) {
        const RowSplit rs = row_split(p, r, total, ctas);
        if (rs.first == rs.last) store_out<NB>(p, y, r * 128 + rit0, q);
        else publish_partial<NB>(p, cta, r == first_row ? 0 : 1, y, rit0, q);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) y[nb][e] = 0.0f;
      }
    }
  }
}

// --------------------------------------------------------------------------------------
// Uniform-depth streaming GEMV: the same per-warp streaming as gemv_stream_kernel with
// the depth D a compile-time constant.  The plane is tile-major, so the CTA walks
// consecutive tile indices (the next tile is always +4352 bytes, also across a tile
// row) and each tile's D stages become D independent tensor-core chains.  kTilesAhead
// tiles of records are kept in flight in registers.  With I8 (batch <= 2) the
// chains are integer m16n8k32 MMAs on int8 activation limbs (4 per tile-stage instead
// of 8 FP16 MMAs, and 16 ANDs of decode instead of 32 ANDs and 4 shifts).

template <int D>
struct TilesAhead {
  static constexpr int value = D == 1 ? 8 : (D == 2 ? 4 : (D == 3 ? 3 : 2));
};

// Per-lane byte offsets of the activation data inside one tile slot.  Lanes whose batch
// row does not exist read the last real row instead: their MMA columns and epilogue
// values are never stored, and copies of real data keep them finite.
template <int NB, int XL>
struct XLane {
  uint32_t frag[NB];    // B-fragment row of batch g + 8*nb (first of XL halves)
  uint32_t fg[NB][2];   // {factor, correction} of batch 2q + j + 8*nb
  uint32_t half_stride; // bytes between the XL halves (batch * 256)

  __device__ __forceinline__ XLane(uint32_t batch, uint32_t lane) {
    const uint32_t g = lane >> 2, q = lane & 3;
    half_stride = batch * 256;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const uint32_t b = min(g + 8 * nb, batch - 1);
      frag[nb] = (b * 4 + q) * 64;
#pragma unroll
      for (int j = 0; j < 2; ++j) fg[nb][j] = batch * 256 * XL + min(2 * q + j + 8 * nb, batch - 1) * 8;
    }
  }
};

template <int NB, int XL>
__device__ __forceinline__ void load_xfrag(XFrag<NB, XL>& xf, const XLane<NB, XL>& xl, const uint8_t* slot) {
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
    for (int l = 0; l < XL; ++l) {
      const uint8_t* src = slot + xl.frag[nb] + l * xl.half_stride;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 t = lds128(src + 16 * v);
        xf.bf[nb][l][2 * v][0] = t.x;
        xf.bf[nb][l][2 * v][1] = t.y;
        xf.bf[nb][l][2 * v + 1][0] = t.z;
        xf.bf[nb][l][2 * v + 1][1] = t.w;
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 fg = lds_f2(slot + xl.fg[nb][j]);
      xf.f[nb][j] = fg.x;
      xf.gsum[nb][j] = fg.y;
    }
  }
}

// One lane's part of one row block of a plane record: its 16-byte code slot and its
// 4-byte scale pair, read once (no L1 allocation) and marked evict-first in L2, so the
// streamed planes do not push activations and other reused data out of L2.
__device__ __forceinline__ void ld_plane(uint4& w, uint32_t& sc, const uint8_t* codes, const uint8_t* scales,
                                         uint64_t policy) {
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
               : "l"(codes), "l"(policy));
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(sc) : "l"(scales), "l"(policy));
}


// Tensor-core part of one tile (its D stage records w): D independent MMA chains (two
// for D == 1); the first MMA of each chain starts from zero.
template <int NB, int XL, int D>
__device__ __forceinline__ void tile_mma(const uint4 (&w)[D], const XFrag<NB, XL>& xf, uint32_t shift_mul,
                                         float (&acc)[TileChains<D>::value][NB][4]) {
  uint32_t hi[D][4];
#pragma unroll
  for (int s = 0; s < D; ++s) {
    hi[s][0] = __umulhi(w[s].x, shift_mul);
    hi[s][1] = __umulhi(w[s].y, shift_mul);
    hi[s][2] = __umulhi(w[s].z, shift_mul);
    hi[s][3] = __umulhi(w[s].w, shift_mul);
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
#pragma unroll
    for (int s = 0; s < D; ++s) {
      const int c = D == 1 ? (m & 1) : s;
      const bool first = D == 1 ? m < 2 : m == 0;
      const uint32_t a0 = int2_pair(w[s].x, hi[s][0], m), a1 = int2_pair(w[s].y, hi[s][1], m);
      const uint32_t a2 = int2_pair(w[s].z, hi[s][2], m), a3 = int2_pair(w[s].w, hi[s][3], m);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int l = 0; l < XL; ++l) {
          if (first && l == 0) mma_f16_zero(acc[c][nb], a0, a1, a2, a3, xf.bf[nb][l][m][0], xf.bf[nb][l][m][1]);
          else mma_f16(acc[c][nb], a0, a1, a2, a3, xf.bf[nb][l][m][0], xf.bf[nb][l][m][1]);
        }
    }
  }
}

// Scale epilogue of one tile into y: y += σ·(acc·2^(24+e) − 2^(e+1)·Σx̃) per stage.
// With B1 (batch 1) only accumulator column 0 is ever stored: the others are skipped.
template <int NB, int XL, int D, bool B1>
__device__ __forceinline__ void tile_epilogue(const uint32_t (&sc)[D], const XFrag<NB, XL>& xf,
                                              float (&acc)[TileChains<D>::value][NB][4], float (&y)[NB][4]) {
  constexpr int CH = TileChains<D>::value;
  if (D == 1) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      acc[0][nb][0] += acc[CH - 1][nb][0];
      acc[0][nb][2] += acc[CH - 1][nb][2];
      if (!B1) {
        acc[0][nb][1] += acc[CH - 1][nb][1];
        acc[0][nb][3] += acc[CH - 1][nb][3];
      }
    }
  }
#pragma unroll
  for (int s = 0; s < D; ++s) {
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sc[s]);
    const float s_lo = __low2float(s2), s_hi = __high2float(s2);
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      y[nb][0] = fmaf(s_lo, fmaf(acc[s][nb][0], xf.f[nb][0], -xf.gsum[nb][0]), y[nb][0]);
      y[nb][2] = fmaf(s_hi, fmaf(acc[s][nb][2], xf.f[nb][0], -xf.gsum[nb][0]), y[nb][2]);
      if (!B1) {
        y[nb][1] = fmaf(s_lo, fmaf(acc[s][nb][1], xf.f[nb][1], -xf.gsum[nb][1]), y[nb][1]);
        y[nb][3] = fmaf(s_hi, fmaf(acc[s][nb][3], xf.f[nb][1], -xf.gsum[nb][1]), y[nb][3]);
      }
    }
  }
}


template <int XL>
__device__ __forceinline__ void build_xfrag_tiles(const GemvParams& p, uint8_t* xres, const ColRanges& cr,
                                                  uint32_t c_first) {
  using XT = typename std::conditional<XL == 1, __half, float>::type;
  const XT* x = static_cast<const XT*>(p.x_raw);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = 2;
  constexpr uint32_t kWarps = kStreamThreads / 32;
  const uint32_t items = cr.count() * p.batch;
  for (uint32_t base = warp; base < items; base += W * kWarps) {
    float v[W][4];
    bool ok[W];
    uint8_t* slot[W];
    uint32_t b[W];
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const uint32_t item = base + w * kWarps;
      ok[w] = item < items;
      const uint32_t it = ok[w] ? item : base;
      const uint32_t ci = it / p.batch;
      b[w] = it - ci * p.batch;
      const uint32_t c = cr.col(ci);
      slot[w] = xres + resident_slot(c, c_first, p.C) * p.xslot_bytes;
      load_x4<XT>(x + static_cast<uint64_t>(b[w]) * p.cols, c * 128 + 4 * lane, p.cols, p.x_vec != 0, v[w]);
    }
    prep_items<XL, W>(v, ok, slot, b, p.batch, lane);
  }
}

// The stream-K kernel's work on FP16 fragments as CTA `cta` of a grid of `grid` CTAs on
// problem p (int8 limb launches run lean_body or unit_body instead).
template <int NB, int XL, int D, bool B1 = false>
__device__ __forceinline__ void uniform_body(const GemvParams& p, const uint32_t cta, const uint32_t grid) {
  constexpr int R = TilesAhead<D>::value;
  constexpr uint32_t kFull = (1u << D) - 1u;
  extern __shared__ __align__(16) uint8_t xres[];  // [resident activation slots]
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  // The CTA's units [u0, u1): tiles t0..t_end, the first from stage s0, the last up to
  // stage s_end; rb_first / re_last: first unit of t0's tile row, end of t_end's.
  MixedRange rg{};
  rg.total = p.total;
  rg.ctas = static_cast<uint32_t>(rg.total < grid ? rg.total : grid);
  if (cta < rg.ctas) {
    rg.u0 = unit_start(cta, rg.total, rg.ctas);
    rg.u1 = unit_start(cta + 1, rg.total, rg.ctas);
    rg.t0 = static_cast<uint32_t>(rg.u0 / D);
    rg.s0 = static_cast<uint32_t>(rg.u0 % D);
    rg.t_end = static_cast<uint32_t>((rg.u1 - 1) / D);
    rg.s_end = static_cast<uint32_t>((rg.u1 - 1) % D) + 1;
    rg.rb_first = static_cast<uint64_t>(rg.t0 / p.C) * p.C * D;
    rg.re_last = static_cast<uint64_t>(rg.t_end / p.C + 1) * p.C * D;
  }
  const uint64_t total = rg.total, u0 = rg.u0, u1 = rg.u1;
  const uint32_t ctas = rg.ctas;
  griddep_launch_dependents();  // a following PDL kernel may be scheduled; it waits for this grid
  if (cta >= ctas) return;
  const uint32_t rit0 = warp * 16 + g;
  const uint32_t t0 = rg.t0, s0 = rg.s0, t_end = rg.t_end, s_end = rg.s_end;
  const uint32_t ntiles = t_end - t0 + 1;
  const uint32_t mask_first = kFull & ~((1u << s0) - 1u), mask_last = (1u << s_end) - 1u;
  // Stages of walk tile k (tile t_end - k) this CTA computes: all D, cut to the range at
  // its two ends.
  auto tile_mask = [&](uint32_t k) -> uint32_t {
    uint32_t m = kFull;
    if (k == 0) m &= mask_last;
    if (k == ntiles - 1) m &= mask_first;
    return m;
  };
  // The CTA walks its tiles in descending order: its last tile row, which goes on in the
  // next CTA, comes first and its part is published early; its first row, which it sums
  // when that row began in an earlier CTA, comes last.
  // Per-stage code and scale pointers of this lane, at the first tile of the group of R
  // tiles that the next refills load; slot j of a group is at -j*4352 bytes.
  // Deep prefixes derive the scale address from the code address (fewer registers).
  constexpr bool kScalePtr = D <= 2;
  constexpr int SB = kScalePtr ? D : 1;
  const uint8_t* cb[D];
  const uint8_t* sb[SB];
  const uint32_t lane_off = warp * kRowBlockBytes + lane * 16, scale_off = warp * kRowBlockBytes + 512 + g * 4;
  const uint32_t scale_rel = scale_off - lane_off;
#pragma unroll
  for (int s = 0; s < D; ++s) {
    cb[s] = p.planes[s] + static_cast<uint64_t>(t_end) * kRecordBytes + lane_off;
    if (kScalePtr) sb[s < SB ? s : 0] = p.planes[s] + static_cast<uint64_t>(t_end) * kRecordBytes + scale_off;
  }

  // Register ring of R tiles x D stages.  A stage outside the CTA's units gets scale 0
  // (codes 0): its products are finite and its contribution is exactly zero.
  uint4 w[R][D];
  uint32_t sc[R][D];
  const uint64_t l2_first = policy_evict_first();
  auto load_tile = [&](int slot, uint32_t mask) {
#pragma unroll
    for (int s = 0; s < D; ++s) {
      if (D == 1 || (mask & (1u << s))) {
        const uint8_t* a = cb[s] - slot * kRecordBytes;
        const uint8_t* as = kScalePtr ? sb[s < SB ? s : 0] - slot * kRecordBytes : a + scale_rel;
        ld_plane(w[slot][s], sc[slot][s], a, as, l2_first);
      } else {
        w[slot][s] = make_uint4(0u, 0u, 0u, 0u);
        sc[slot][s] = 0u;
      }
    }
  };
  auto next_group = [&]() {
#pragma unroll
    for (int s = 0; s < D; ++s) {
      cb[s] -= R * kRecordBytes;
      if (kScalePtr) sb[s < SB ? s : 0] -= R * kRecordBytes;
    }
  };
#pragma unroll
  for (int j = 0; j < R; ++j) {
    if (static_cast<uint32_t>(j) < ntiles) load_tile(j, tile_mask(j));
  }
  next_group();
  griddep_wait();
  const uint32_t c_first = t0 % p.C;
  if (min(p.C, ntiles) > p.x_res_slots) {  // the launch sized shared memory for fewer slots
    if (threadIdx.x == 0) atomicOr(p.error, HQB_DEVERR_LAUNCH);
    return;
  }
  {  // activation fragments of the tile columns this CTA touches, at their resident slots
    const ColRanges cr = needed_columns(t0, t_end, p.C);
    if (p.x_raw != nullptr) {
      build_xfrag_tiles<XL>(p, xres, cr, c_first);
    } else {
      const uint32_t per_slot = p.xslot_bytes / 16;
      const uint32_t chunks = cr.count() * per_slot;
      for (uint32_t t = threadIdx.x; t < chunks; t += kStreamThreads) {
        const uint32_t ci = t / per_slot, k = t - ci * per_slot, c = cr.col(ci);
        const uint4* src = reinterpret_cast<const uint4*>(p.xfrag + static_cast<uint64_t>(c) * p.xslot_bytes) + k;
        reinterpret_cast<uint4*>(xres + resident_slot(c, c_first, p.C) * p.xslot_bytes)[k] = __ldcg(src);
      }
    }
  }
  __syncthreads();
  const XLane<NB, XL> xlane(p.batch, lane);
  uint32_t row = t_end / p.C;
  // activation slot of the current tile; the next tile's is the previous slot (mod C)
  const uint8_t* xs = xres + resident_slot(t_end % p.C, c_first, p.C) * p.xslot_bytes;
  const uint8_t* const xs_top = xres + (p.C - 1) * p.xslot_bytes;
  uint32_t left = t_end % p.C + 1;  // tiles of the current row still ahead (may run past ntiles)
  float y[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) y[nb][e] = 0.0f;

  constexpr int CH = TileChains<D>::value;
  // After tile k: the row may end (its column 0, or the CTA's last tile).  A row wholly
  // inside the range is stored; one that goes on in later CTAs is published; the CTA's
  // first row, when it began in an earlier CTA and ends here, is kept and summed after
  // the last tile.
  float kept[NB][4];
  bool keep = false;
  const uint32_t row_first = t0 / p.C, row_last = t_end / p.C;
  auto advance = [&](uint32_t k) {
    if (--left == 0 || k + 1 == ntiles) {
      // the row's unit range, as far as it matters: inside [u0, u1) unless an end row
      const uint64_t rb = row == row_first ? rg.rb_first : u0, re = row == row_last ? rg.re_last : u1;
      if (rb >= u0 && re <= u1) {
        store_out<NB>(p, y, row * 128 + rit0, q);
      } else if (re > u1) {
        publish_flagged<NB>(p, cta, y, rit0, q);
      } else {
        keep = true;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
          for (int e = 0; e < 4; ++e) kept[nb][e] = y[nb][e];
      }
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) y[nb][e] = 0.0f;
      --row;
      left = p.C;
    }
    xs = xs == xres ? xs_top : xs - p.xslot_bytes;
  };
  auto one_tile = [&](int j) {
    XFrag<NB, XL> xf;
    load_xfrag<NB, XL>(xf, xlane, xs);
    float acc[CH][NB][4];
    tile_mma<NB, XL, D>(w[j], xf, p.shift_mul, acc);
    tile_epilogue<NB, XL, D, B1>(sc[j], xf, acc, y);
  };

  uint32_t k0 = 0;
  for (; k0 + R <= ntiles; k0 += R) {  // whole groups of R tiles
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const uint32_t k = k0 + j;
      one_tile(j);
      const uint32_t kn = k + R;  // refill slot j with tile kn (group base cb/sb)
      if (kn < ntiles) load_tile(j, tile_mask(kn));
      advance(k);
    }
    next_group();
  }
#pragma unroll
  for (int j = 0; j < R; ++j) {  // the last partial group (no more loads)
    const uint32_t k = k0 + j;
    if (k >= ntiles) break;
    one_tile(j);
    advance(k);
  }
  if (keep) reduce_split_row<NB, B1>(p, row_first, rg.rb_first, total, ctas, cta, kept, rit0, q);
  if (p.g_world > 1) gather_signal(p, ctas);
}

// The stream-K kernel's int8-limb form at a uniform prefix, written for the fewest
// instructions per (row block, stage) task: the same partition, descending walk, register
// ring, split-row scheme and arithmetic as uniform_body, with
//   * the steady-state loop over whole groups of R tiles whose refills are interior tiles:
//     every refill loads all D stage records with no mask and no bound test;
//   * the CTA's two edge tiles (partial stage ranges) loaded with masks, outside that loop;
//   * MMA chains from zero (the 1.5·2^23 bias added in the epilogue), limb slots at 32-bit
//     shared addresses, and limb slots built by limb_item (so activations up to the FP32
//     maximum keep the contract, and a NaN or Inf gives NaN outputs).
// Shared memory: the resident limb slots, then a 512-byte transpose area per warp.
template <int XL, int D, bool B1>
__device__ __forceinline__ void lean_body(const GemvParams& p, const uint32_t cta, const uint32_t grid) {
  constexpr int R = TilesAhead<D>::value;
  constexpr uint32_t kFull = (1u << D) - 1u;
  constexpr int CH = TileChains<D>::value;
  constexpr uint32_t XS = kLimbs * (B1 ? 1u : 2u) * 128u + 80u;  // xslot_i8_bytes(batch)
  constexpr uint32_t kWideOff = kLimbs * (B1 ? 1u : 2u) * 128u + 64u;
  extern __shared__ __align__(16) uint8_t xres[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const uint64_t total = p.total;
  const uint32_t ctas = static_cast<uint32_t>(total < grid ? total : grid);
  griddep_launch_dependents();  // a following PDL kernel may be scheduled; it waits for this grid
  if (cta >= ctas) return;
  uint64_t u0, u1;
  if (total * (ctas + 1ull) <= 0xffffffffull) {  // 32-bit divisions (the usual case)
    const uint32_t T = static_cast<uint32_t>(total);
    u0 = (cta * T) / ctas;
    u1 = ((cta + 1) * T) / ctas;
  } else {
    u0 = unit_start(cta, total, ctas);
    u1 = unit_start(cta + 1, total, ctas);
  }
  const uint32_t C = p.C;
  const uint32_t t0 = static_cast<uint32_t>(u0 / D), s0 = static_cast<uint32_t>(u0 % D);
  const uint32_t t_end = static_cast<uint32_t>((u1 - 1) / D), s_end = static_cast<uint32_t>((u1 - 1) % D) + 1;
  const uint32_t row_first = t0 / C, row_last = t_end / C;
  const uint64_t rb_first = static_cast<uint64_t>(row_first) * C * D;
  const uint64_t re_last = static_cast<uint64_t>(row_last + 1) * C * D;
  const uint32_t ntiles = t_end - t0 + 1;
  const uint32_t mask_first = kFull & ~((1u << s0) - 1u), mask_last = (1u << s_end) - 1u;
  const uint32_t rit0 = warp * 16 + g;

  // Records of walk tile k (tile t_end - k) for this lane: cb[s] - k * 4352 (codes), the
  // scale pair scale_rel bytes further.  cur[s] points at the first tile the next group's
  // refills load (walk tile k0 + R), so refill j of a group is cur[s] - j * 4352.
  const uint32_t lane_off = warp * kRowBlockBytes + lane * 16;
  const uint32_t scale_rel = 512 + g * 4 - lane * 16;
  const uint64_t l2_first = policy_evict_first();
  const uint8_t* base[D];
#pragma unroll
  for (int s = 0; s < D; ++s) base[s] = p.planes[s] + static_cast<uint64_t>(t_end) * kRecordBytes + lane_off;
  uint4 w[R][D];
  uint32_t sc[R][D];
  // walk tile k into ring slot `slot`; stages outside `mask` are not loaded and read as
  // scale 0 with codes 0 (their products are exactly zero)
  auto load_masked = [&](int slot, uint32_t k, uint32_t mask) {
#pragma unroll
    for (int s = 0; s < D; ++s) {
      if (mask & (1u << s)) {
        const uint8_t* a = base[s] - static_cast<uint64_t>(k) * kRecordBytes;
        ld_plane(w[slot][s], sc[slot][s], a, a + scale_rel, l2_first);
      } else {
        w[slot][s] = make_uint4(0u, 0u, 0u, 0u);
        sc[slot][s] = 0u;
      }
    }
  };
  auto edge_mask = [&](uint32_t k) -> uint32_t {
    uint32_t m = kFull;
    if (k == 0) m &= mask_last;
    if (k == ntiles - 1) m &= mask_first;
    return m;
  };
#pragma unroll
  for (int j = 0; j < R; ++j)
    if (static_cast<uint32_t>(j) < ntiles) load_masked(j, j, edge_mask(j));
  griddep_wait();
  const uint32_t c_first = t0 % C;
  if (min(C, ntiles) > p.x_res_slots) {  // the launch sized shared memory for fewer slots
    if (threadIdx.x == 0) atomicOr(p.error, HQB_DEVERR_LAUNCH);
    return;
  }
  {
    const ColRanges cr = needed_columns(t0, t_end, C);
    if (p.x_raw != nullptr) {
      build_limb_slots<XL, kStreamThreads / 32>(p, xres,
                                                reinterpret_cast<float*>(xres + p.x_res_slots * XS) + warp * 128, cr,
                                                c_first, warp, lane);
    } else {  // slots prepared by one launch for all CTAs (prep_limbs_kernel)
      constexpr uint32_t per_slot = XS / 16;
      const uint32_t chunks = cr.count() * per_slot;
      for (uint32_t t = threadIdx.x; t < chunks; t += kStreamThreads) {
        const uint32_t ci = t / per_slot, k = t - ci * per_slot, c = cr.col(ci);
        const uint4* src = reinterpret_cast<const uint4*>(p.xfrag + static_cast<uint64_t>(c) * XS) + k;
        reinterpret_cast<uint4*>(xres + resident_slot(c, c_first, C) * XS)[k] = __ldcg(src);
      }
    }
  }
  __syncthreads();

  const XLaneI8 xl8(B1 ? 1u : 2u, lane);
  const uint32_t xres_a = smem_u32(xres);
  const uint32_t x_top = (C - 1) * XS;
  uint32_t xoff = resident_slot(t_end % C, c_first, C) * XS;  // limb slot of the current tile
  uint32_t row = t_end / C;
  uint32_t left = t_end % C + 1;  // tiles of the current row still ahead (may run past ntiles)
  float y[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  float kept[1][4];
  bool keep = false;

  // Tiles whose limb slot is wide or non-finite (limb_item marks them with K >= 0 or NaN)
  // need the slower epilogue; a CTA without any runs the hot loop without that branch.
  bool any_wide = false;
  {
    const ColRanges cr = needed_columns(t0, t_end, C);
    for (uint32_t i = lane; i < cr.count() * (B1 ? 1u : 2u); i += 32) {
      const uint32_t c = cr.col(B1 ? i : i >> 1), b = B1 ? 0u : (i & 1u);
      const float k = __uint_as_float(lds32a(xres_a + resident_slot(c, c_first, C) * XS + kLimbs * (B1 ? 1u : 2u) * 128u +
                                              (2u * b + 1u) * 4u));
      any_wide = any_wide || !(k < 0.0f);
    }
    any_wide = __any_sync(0xffffffffu, any_wide);
  }

  // The math of the tile in ring slot j (limbs at xres_a + xoff), then the next limb slot.
  // WIDE: the slot may be wide or non-finite (checked per tile).
  auto tile_math = [&](int j, auto wide_tag) {
    constexpr bool WIDE = decltype(wide_tag)::value;
    XFragI8 xf;
    load_limbs<B1>(xf, xres_a + xoff + xl8.frag, xres_a + xoff + xl8.cst);
    uint32_t acc[CH][4];
    bulk_tile_mma<D, false>(w[j], xf, acc, kFull);
    if (!WIDE || (xf.K[0] < 0.0f && (B1 || xf.K[1] < 0.0f))) {
      bulk_tile_epilogue<D, B1, false>(sc[j], xf, acc, y, kFull);
    } else {
      const float f0 = __uint_as_float(lds32a(xres_a + xoff + kWideOff));
      const float f1 = B1 ? 1.0f : __uint_as_float(lds32a(xres_a + xoff + kWideOff + 4));
      bulk_tile_epilogue_wide<D, B1, false>(sc[j], xf, acc, y, kFull, f0, f1);
    }
    xoff = xoff == 0 ? x_top : xoff - XS;
  };
  // End of a tile row (its column 0) or of the CTA's range: the row's sums are stored,
  // published for a later CTA, or kept to be finished last.
  auto flush_row = [&]() {
    quad_sum<B1>(y);
    const uint64_t rb = row == row_first ? rb_first : u0, re = row == row_last ? re_last : u1;
    if (rb >= u0 && re <= u1) {
      store_out<1>(p, y, row * 128 + rit0, q);
    } else if (re > u1) {
      publish_flagged<1>(p, cta, y, rit0, q);
    } else {
      keep = true;
#pragma unroll
      for (int e = 0; e < 4; ++e) kept[0][e] = y[0][e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) y[0][e] = 0.0f;
    --row;
    left = C;
  };

  // Steady state: groups of R tiles k0..k0+R-1 whose refills k0+R..k0+2R-1 are interior
  // tiles (before the CTA's last), so no tile of the group ends the CTA's range.  A group
  // inside one tile row (the usual case) runs with no row-end test; a group that reaches
  // a row end runs tile by tile with it, as a separate block, so the hot loop stays small.
  uint32_t k0 = 0;
  const uint8_t* cur[D];
#pragma unroll
  for (int s = 0; s < D; ++s) cur[s] = base[s] - static_cast<uint64_t>(R) * kRecordBytes;
  auto main_loop = [&](auto wide_tag) {
    for (; k0 + 2 * R < ntiles; k0 += R) {
      if (left > static_cast<uint32_t>(R)) {
#pragma unroll
        for (int j = 0; j < R; ++j) {
          tile_math(j, wide_tag);
#pragma unroll
          for (int s = 0; s < D; ++s) {
            const uint8_t* a = cur[s] - j * kRecordBytes;
            ld_plane(w[j][s], sc[j][s], a, a + scale_rel, l2_first);
          }
        }
        left -= R;
      } else {
#pragma unroll
        for (int j = 0; j < R; ++j) {
          tile_math(j, wide_tag);
#pragma unroll
          for (int s = 0; s < D; ++s) {
            const uint8_t* a = cur[s] - j * kRecordBytes;
            ld_plane(w[j][s], sc[j][s], a, a + scale_rel, l2_first);
          }
          if (--left == 0) flush_row();
        }
      }
#pragma unroll
      for (int s = 0; s < D; ++s) cur[s] -= R * kRecordBytes;
    }
  };
  if (any_wide) main_loop(std::true_type{});
  else main_loop(std::false_type{});
  // The rest (at most 2R tiles): refills with bounds and the edge mask, the CTA's end.
#pragma unroll
  for (int jj = 0; jj < 2 * R; ++jj) {
    const uint32_t k = k0 + jj;
    if (k >= ntiles) break;
    tile_math(jj % R, std::true_type{});
    if (k + R < ntiles) load_masked(jj % R, k + R, edge_mask(k + R));
    if (--left == 0 || k + 1 == ntiles) flush_row();
  }
  if (keep) reduce_split_row<1, B1>(p, row_first, rb_first, total, ctas, cta, kept, rit0, q);
  if (p.g_world > 1) gather_signal(p, ctas);
}

// Per-tile depth maps at batch <= 2 with raw x (or prepared limb slots): the lean body's
// register ring with one (tile, stage) unit per slot, so a warp keeps 8 row-block records
// in flight whatever the depths.  The CTA's units [u0, u1) come from the depth plan
// (mixed_range); the walk goes down the tiles, t_end first, and up the stages inside a
// tile (the uniform kernels' order of stage sums).  The loader runs 8 units ahead of the
// math: it finds each unit's stage plane and tile from the depths (a 32-tile window per
// warp in registers, the next window loaded 32 tiles early) and leaves the math, per slot,
// the unit's limb slot and whether a tile row ends after it.
template <int XL, bool B1>
__device__ __forceinline__ void unit_body(const GemvParams& p, const uint32_t cta) {
  constexpr int R = 8;
  constexpr uint32_t XS = kLimbs * (B1 ? 1u : 2u) * 128u + 80u;  // xslot_i8_bytes(batch)
  constexpr uint32_t kWideOff = kLimbs * (B1 ? 1u : 2u) * 128u + 64u;
  constexpr uint32_t kRowEnd = 0x80000000u;
  extern __shared__ __align__(16) uint8_t xres[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const MixedRange rg = mixed_range(p, cta, lane);
  griddep_launch_dependents();  // a following PDL kernel may be scheduled; it waits for this grid
  if (cta >= rg.ctas) return;
  const uint64_t total = rg.total, u0 = rg.u0, u1 = rg.u1;
  const uint32_t ctas = rg.ctas, C = p.C;
  const uint32_t t0 = rg.t0, s0 = rg.s0, t_end = rg.t_end, s_end = rg.s_end;
  const uint32_t ntiles = t_end - t0 + 1;
  const uint32_t n = static_cast<uint32_t>(u1 - u0);  // this CTA's units
  const uint32_t row_first = t0 / C, row_last = t_end / C;
  const uint64_t rb_first = rg.rb_first, re_last = rg.re_last;
  const uint32_t rit0 = warp * 16 + g;
  const uint32_t c_first = t0 % C;
  const uint32_t lane_off = warp * kRowBlockBytes + lane * 16;
  const uint32_t scale_rel = 512 + g * 4 - lane * 16;
  const uint64_t l2_first = policy_evict_first();
  const uint8_t* pb0 = p.planes[0] + lane_off;
  const uint8_t* pb1 = p.planes[1] + lane_off;
  const uint8_t* pb2 = p.planes[2] + lane_off;
  const uint8_t* pb3 = p.planes[3] + lane_off;

  // Depth window: lane i holds the depth of tile wtop - i (0 below t0).
  auto load_win = [&](uint32_t top) -> uint32_t {
    return (top >= lane && top - lane >= t0) ? clamp_depth(__ldg(p.depth + (top - lane)), p.stage_count) : 0u;
  };
  uint32_t wtop = t_end;
  uint32_t dwin = load_win(wtop);
  uint32_t dnext = wtop >= t0 + 32 ? load_win(wtop - 32) : 0u;
  auto depth_of = [&](uint32_t t) -> uint32_t {  // t = the previous tile asked for, minus one
    if (wtop - t >= 32) {
      wtop -= 32;
      dwin = dnext;
      dnext = wtop >= t0 + 32 ? load_win(wtop - 32) : 0u;
    }
    return __shfl_sync(0xffffffffu, dwin, wtop - t);
  };

  // Loader: the unit the next refill loads (tile lt, stage ls of [.., lend)), its tile
  // column and limb slot offset.
  const uint32_t x_top = (C - 1) * XS;
  uint32_t lt = t_end, ls = t_end == t0 ? s0 : 0u, lend = s_end;
  uint32_t lcol = t_end % C;
  uint32_t lxoff = resident_slot(lcol, c_first, C) * XS;
  uint4 w[R];
  uint32_t sc[R], meta[R];
  auto refill = [&](int j) {
    const uint8_t* b = ls == 0 ? pb0 : (ls == 1 ? pb1 : (ls == 2 ? pb2 : pb3));
    const uint8_t* a = b + static_cast<uint64_t>(lt) * kRecordBytes;
    ld_plane(w[j], sc[j], a, a + scale_rel, l2_first);
    const bool last = ls + 1 == lend;
    meta[j] = lxoff | (last && lcol == 0 ? kRowEnd : 0u);
    if (!last) {
      ++ls;
    } else if (lt > t0) {
      --lt;
      ls = lt == t0 ? s0 : 0u;
      lend = depth_of(lt);
      lxoff = lxoff == 0 ? x_top : lxoff - XS;
      lcol = lcol == 0 ? C - 1 : lcol - 1;
    }
  };
#pragma unroll
  for (int j = 0; j < R; ++j)
    if (static_cast<uint32_t>(j) < n) refill(j);
  griddep_wait();
  if (min(C, ntiles) > p.x_res_slots) {  // the launch sized shared memory for fewer slots
    if (threadIdx.x == 0) atomicOr(p.error, HQB_DEVERR_LAUNCH);
    return;
  }
  const ColRanges cr = needed_columns(t0, t_end, C);
  if (p.x_raw != nullptr) {
    build_limb_slots<XL, kStreamThreads / 32>(p, xres, reinterpret_cast<float*>(xres + p.x_res_slots * XS) + warp * 128,
                                              cr, c_first, warp, lane);
  } else {  // slots prepared by one launch for all CTAs (prep_limbs_kernel)
    constexpr uint32_t per_slot = XS / 16;
    const uint32_t chunks = cr.count() * per_slot;
    for (uint32_t t = threadIdx.x; t < chunks; t += kStreamThreads) {
      const uint32_t ci = t / per_slot, k = t - ci * per_slot, c = cr.col(ci);
      const uint4* src = reinterpret_cast<const uint4*>(p.xfrag + static_cast<uint64_t>(c) * XS) + k;
      reinterpret_cast<uint4*>(xres + resident_slot(c, c_first, C) * XS)[k] = __ldcg(src);
    }
  }
  __syncthreads();

  const XLaneI8 xl8(B1 ? 1u : 2u, lane);
  const uint32_t xres_a = smem_u32(xres);
  bool any_wide = false;
  for (uint32_t i = lane; i < cr.count() * (B1 ? 1u : 2u); i += 32) {
    const uint32_t c = cr.col(B1 ? i : i >> 1), b = B1 ? 0u : (i & 1u);
    const float k = __uint_as_float(
        lds32a(xres_a + resident_slot(c, c_first, C) * XS + kLimbs * (B1 ? 1u : 2u) * 128u + (2u * b + 1u) * 4u));
    any_wide = any_wide || !(k < 0.0f);
  }
  any_wide = __any_sync(0xffffffffu, any_wide);

  uint32_t row = t_end / C;
  float y[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  float kept[1][4];
  bool keep = false;
  auto unit_math = [&](int j, uint32_t xo, auto wide_tag) {
    constexpr bool WIDE = decltype(wide_tag)::value;
    XFragI8 xf;
    load_limbs<B1>(xf, xres_a + xo + xl8.frag, xres_a + xo + xl8.cst);
    uint32_t acc[2][4];
    const uint4(&wj)[1] = *reinterpret_cast<const uint4(*)[1]>(&w[j]);
    const uint32_t(&sj)[1] = *reinterpret_cast<const uint32_t(*)[1]>(&sc[j]);
    bulk_tile_mma<1, false>(wj, xf, acc, 1u);
    if (!WIDE || (xf.K[0] < 0.0f && (B1 || xf.K[1] < 0.0f))) {
      bulk_tile_epilogue<1, B1, false>(sj, xf, acc, y, 1u);
    } else {
      const float f0 = __uint_as_float(lds32a(xres_a + xo + kWideOff));
      const float f1 = B1 ? 1.0f : __uint_as_float(lds32a(xres_a + xo + kWideOff + 4));
      bulk_tile_epilogue_wide<1, B1, false>(sj, xf, acc, y, 1u, f0, f1);
    }
  };
  auto flush_row = [&]() {
    quad_sum<B1>(y);
    const uint64_t rb = row == row_first ? rb_first : u0, re = row == row_last ? re_last : u1;
    if (rb >= u0 && re <= u1) {
      store_out<1>(p, y, row * 128 + rit0, q);
    } else if (re > u1) {
      publish_flagged<1>(p, cta, y, rit0, q);
    } else {
      keep = true;
#pragma unroll
      for (int e = 0; e < 4; ++e) kept[0][e] = y[0][e];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) y[0][e] = 0.0f;
    --row;
  };

  // Steady state: groups of R units whose refills are all units of this CTA (no tests but
  // the row end); then the rest, refilled only where a unit remains R ahead (no unit needs a
  // mask, so the rest is the same loop with those tests).
  auto main_loop = [&](auto wide_tag) {
    uint32_t k0 = 0;
    for (; k0 + 2 * R <= n; k0 += R) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const uint32_t m = meta[j];
        unit_math(j, m & ~kRowEnd, wide_tag);
        refill(j);
        if (m & kRowEnd) flush_row();
      }
    }
    for (; k0 < n; k0 += R) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const uint32_t k = k0 + j;
        if (k >= n) break;
        const uint32_t m = meta[j];
        unit_math(j, m & ~kRowEnd, wide_tag);
        if (k + R < n) refill(j);
        if ((m & kRowEnd) || k + 1 == n) flush_row();
      }
    }
  };
  if (any_wide) main_loop(std::true_type{});
  else main_loop(std::false_type{});
  if (keep) reduce_split_row<1, B1>(p, row_first, rb_first, total, ctas, cta, kept, rit0, q);
  if (p.g_world > 1) gather_signal(p, ctas);
}

template <int XL, bool B1>
__global__ void __launch_bounds__(kStreamThreads, 2) gemv_unit_kernel(const __grid_constant__ GemvParams p) {
  unit_body<XL, B1>(p, blockIdx.x);
}

template <int NB, int XL, int D, bool B1 = false, bool I8 = false>
__global__ void __launch_bounds__(kStreamThreads, (NB == 1 && (XL == 1 || I8)) ? 2 : 1)
    gemv_uniform_kernel(const __grid_constant__ GemvParams p) {
  static_assert(!I8 || NB == 1, "the int8 limb path takes batch <= 2");
  if constexpr (I8) lean_body<XL, D, B1>(p, blockIdx.x, gridDim.x);
  else uniform_body<NB, XL, D, B1>(p, blockIdx.x, gridDim.x);
}

// Independent GEMVs in one launch (hqb_gemv_grouped): CTAs [cta_base[k], cta_base[k+1]) run
// problem k's stream-K share, so every problem streams at once and the launch's fixed costs
// (start, activation limbs, tail) are paid once for the group.
constexpr uint32_t kMaxGroup = 8;
// Streaming time of building one limb column in a CTA, in (tile, stage) units.  Per-CTA
// timelines of the 7B block step suggest ~1.3 (~0.2 us per column against ~0.156 us per
// unit at two CTAs per SM); timed on B200, 0.8 gives the fastest 7B block step (27.8 against
// 28.6 us at 1.3 and 2.0) and the 70B MLP step of the unweighted dealing (1.3: 2 % faster).
constexpr double kLimbColUnits = 0.8;
struct GroupParams {
  GemvParams p[kMaxGroup];
  uint32_t cta_base[kMaxGroup + 1];
  uint32_t count;
};
static_assert(sizeof(GroupParams) <= 4096, "kernel parameter space");

template <int XL, int D, bool B1>
__global__ void __launch_bounds__(kStreamThreads, 2) gemv_grouped_kernel(const __grid_constant__ GroupParams g) {
  uint32_t k = 0;
  while (k + 1 < g.count && blockIdx.x >= g.cta_base[k + 1]) ++k;
  lean_body<XL, D, B1>(g.p[k], blockIdx.x - g.cta_base[k], g.cta_base[k + 1] - g.cta_base[k]);
}

// --------------------------------------------------------------------------------------
// Row-block GEMV (uniform depth, batch <= 8): the default for a uniform prefix.
//
// Work item: row block b (16 output rows) of tile row r across all C tiles and the D
// selected stages, item index 8r + b.  CTA c (one CTA of kRowsWarps warps per SM) takes
// items c, c + G, c + 2G, ...; the 8 row blocks of a tile row go to 8 consecutive CTAs,
// which together read whole tile records at about the same time.  An item's C·D
// (tile, stage) units are split over the warps in contiguous ranges, the same range for
// every item, so a warp needs the activation fragments of the same few tile columns
// throughout and prepares them once, in its own shared-memory area.
//
// At the end of its range of an item a warp stores its partial sums (16 rows x batch)
// into a shared-memory slot and signals a named barrier without waiting (bar.arrive);
// the item's reducer warp (item j: warp j % 16, which spreads the waiting) completes the
// barrier with bar.sync, adds the parts in warp order, adds the bias and stores the
// rows.  No memory fence is needed, so the register prefetch of the other warps stays in
// flight, and no tile row is split between CTAs, so no partial sums travel through
// global memory.  Reduction slots (one named barrier each) alternate between items; a
// warp that gets kRedSlots items ahead waits (bounded) until the older item is summed.

constexpr uint32_t kRowsWarps = 16;
constexpr uint32_t kRowsThreads = kRowsWarps * 32;
constexpr uint32_t kRedSlots = 2;
constexpr uint32_t kRedSlotFloats = kRowsWarps * 16 * 8;  // [warp][row 0..15][batch 0..7]
constexpr uint32_t kRowsHeadBytes = kRedSlots * kRedSlotFloats * 4 + 256;
constexpr uint32_t kRowsSmemMax = 200 * 1024;
constexpr uint32_t kRowsUnitsMax = 16;  // size rule of the default kernel choice

// First unit of warp w's range among the U units of an item.
__host__ __device__ inline uint32_t rows_unit_start(uint32_t w, uint32_t U) {
  return static_cast<uint32_t>(static_cast<uint64_t>(w) * U / kRowsWarps);
}

template <int XL, int D, bool B1, bool I8 = false>
__global__ void __launch_bounds__(kRowsThreads, 1) gemv_rows_kernel(const __grid_constant__ GemvParams p) {
  using XT = typename std::conditional<XL == 1, __half, float>::type;
  constexpr int R = TilesAhead<D>::value;
  constexpr int CH = TileChains<D>::value;
  constexpr uint32_t kFull = (1u << D) - 1u;
  extern __shared__ __align__(128) uint8_t smem[];
  // [kRedSlots][kRowsWarps][16][8] partial sums | slot generations | fragments
  float* red = reinterpret_cast<float*>(smem);
  volatile uint32_t* gen = reinterpret_cast<uint32_t*>(smem + kRedSlots * kRedSlotFloats * 4);
  volatile uint32_t* gave_up = gen + kRedSlots;  // a slot wait timed out: no warp waits again
  griddep_launch_dependents();  // a following PDL kernel may be scheduled; it waits for this grid
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const uint32_t C = p.C, U = C * D, G = gridDim.x, cta = blockIdx.x;
  const uint32_t items = p.R * 8;
  const uint32_t n_items = cta < items ? (items - cta - 1) / G + 1 : 0;
  // this warp's units [ua, ub) of every item: tiles ta..te, the first and last partial
  const uint32_t ua = rows_unit_start(warp, U), ub = rows_unit_start(warp + 1, U);
  uint32_t ta = 0, te = 0, mask_first = kFull, mask_last = kFull;
  if (ua < ub) {
    ta = ua / D;
    te = (ub - 1) / D;
    mask_first = kFull & ~((1u << (ua % D)) - 1u);
    mask_last = (1u << ((ub - 1) % D + 1)) - 1u;
  }
  const uint32_t nt = te - ta + 1;
  const uint32_t total = ua < ub ? n_items * nt : 0;  // tiles this warp streams
  // byte offset of this lane's code slot in tile column ta of item i (planes < 4 GiB)
  const uint32_t scale_rel = 512 + g * 4 - lane * 16;
  auto item_off = [&](uint32_t i) -> uint32_t {
    return ((i >> 3) * C + ta) * kRecordBytes + (i & 7) * kRowBlockBytes + lane * 16;
  };

  // Register ring of R tiles x D stages, filled in the warp's tile order.  A stage
  // outside the warp's units gets scale 0 (codes 0): it contributes exactly zero.
  uint4 w[R][D];
  uint32_t sc[R][D];
  const uint64_t l2_first = policy_evict_first();
  uint32_t lt = ta, lj = 0;  // next tile to load: column lt of the CTA's item lj
  uint32_t loff = item_off(cta);  // its code-slot offset
  auto load_next = [&](int slot) {
    const uint32_t mask = (lt == ta ? mask_first : kFull) & (lt == te ? mask_last : kFull);
    const uint32_t soff = loff + scale_rel;
#pragma unroll
    for (int s = 0; s < D; ++s) {
      if (D == 1 || (mask & (1u << s))) {
        ld_plane(w[slot][s], sc[slot][s], p.planes[s] + loff, p.planes[s] + soff, l2_first);
      } else {
        w[slot][s] = make_uint4(0u, 0u, 0u, 0u);
        sc[slot][s] = 0u;
      }
    }
    if (++lt > te) {
      lt = ta;
      ++lj;
      loff = item_off(cta + lj * G);
    } else {
      loff += kRecordBytes;
    }
  };
#pragma unroll
  for (int j = 0; j < R; ++j)
    if (static_cast<uint32_t>(j) < total) load_next(j);
  if (threadIdx.x < kRedSlots) gen[threadIdx.x] = threadIdx.x;
  if (threadIdx.x == 0) *gave_up = 0u;
  __syncthreads();
  griddep_wait();

  // activation fragments of tile columns ta..te, in this warp's own area
  uint8_t* xw = smem + kRowsHeadBytes + warp * p.xw_bytes;
  if (total != 0) {
    if (p.x_raw != nullptr) {
      const XT* x = static_cast<const XT*>(p.x_raw);
      const uint32_t n = nt * p.batch;
      for (uint32_t base = 0; base < n; base += 2) {
        float v[2][4];
        bool ok[2];
        uint8_t* slot[2];
        uint32_t b[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          ok[i] = base + i < n;
          const uint32_t it = ok[i] ? base + i : base;
          const uint32_t t = B1 ? it : it / p.batch;
          b[i] = it - t * p.batch;
          slot[i] = xw + t * p.xslot_bytes;
          load_x4<XT>(x + static_cast<uint64_t>(b[i]) * p.cols, (ta + t) * 128 + 4 * lane, p.cols, p.x_vec != 0,
                      v[i]);
        }
        if constexpr (I8) prep_i8_items<2>(v, ok, slot, b, p.batch, lane);
        else prep_items<XL, 2>(v, ok, slot, b, p.batch, lane);
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(p.xfrag + static_cast<uint64_t>(ta) * p.xslot_bytes);
      uint4* dst = reinterpret_cast<uint4*>(xw);
      const uint32_t chunks = nt * p.xslot_bytes / 16;
      for (uint32_t k = lane; k < chunks; k += 32) dst[k] = __ldcg(src + k);
    }
    __syncwarp();
  }

  // warps with a non-empty range take part in every item; with fewer units than warps
  // warp 15 (whose range is never empty) reduces every item
  uint32_t members = 0;
#pragma unroll
  for (uint32_t k = 0; k < kRowsWarps; ++k)
    if (rows_unit_start(k, U) < rows_unit_start(k + 1, U)) members |= 1u << k;
  const uint32_t bar_threads = 32u * __popc(members);
  const bool all_members = U >= kRowsWarps;

  const XLane<1, XL> xlane(p.batch, lane);
  const XLaneI8 xlane8(p.batch, lane);
  float y[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  uint32_t ct = ta, cj = 0;  // tile being computed: column ct of the CTA's item cj
  const uint8_t* xs = xw;

  // End of this warp's range of item j: publish its part; the item's reducer sums.
  auto finish_item = [&](uint32_t j) {
    const uint32_t s = j & (kRedSlots - 1);
    if (lane == 0 && gen[s] != j && *gave_up == 0u) {  // free once item j - kRedSlots is summed
      const unsigned long long t0 = global_timer_ns();
      while (gen[s] != j) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(p.error, HQB_DEVERR_TIMEOUT);
          *gave_up = 1u;
          break;
        }
        __nanosleep(32);
      }
    }
    __syncwarp();
    if constexpr (I8) quad_sum<B1>(y);  // lanes q hold limb columns: every lane gets the sums
    float* part = red + s * kRedSlotFloats;
    if (B1) {
      if (q == 0) {
        part[warp * 16 + g] = y[0][0];
        part[warp * 16 + g + 8] = y[0][2];
      }
    } else {
      float* mine = part + warp * 128;
      *reinterpret_cast<float2*>(mine + g * 8 + 2 * q) = make_float2(y[0][0], y[0][1]);
      *reinterpret_cast<float2*>(mine + (g + 8) * 8 + 2 * q) = make_float2(y[0][2], y[0][3]);
    }
    y[0][0] = y[0][1] = y[0][2] = y[0][3] = 0.0f;
    __syncwarp();
    const uint32_t reducer = all_members ? (j & (kRowsWarps - 1)) : kRowsWarps - 1;
    if (warp != reducer) {
      named_bar_arrive(1 + s, bar_threads);
    } else {
      named_bar_sync(1 + s, bar_threads);
      const uint32_t i = cta + j * G, row0 = (i >> 3) * 128 + (i & 7) * 16;
      for (uint32_t e = lane; e < (B1 ? 16u : 128u); e += 32) {
        const uint32_t rr = B1 ? e : e >> 3, b = B1 ? 0u : e & 7;
        const uint32_t row = row0 + rr;
        if (b >= p.batch || row >= p.rows) continue;
        float sum = 0.0f;
#pragma unroll
        for (uint32_t k = 0; k < kRowsWarps; ++k)
          if (members & (1u << k)) sum += B1 ? part[k * 16 + rr] : part[k * 128 + e];
        if (p.bias != nullptr)
          sum += p.bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(p.bias)[row])
                                         : static_cast<const float*>(p.bias)[row];
        put_y(p, b, row, sum);
      }
      __syncwarp();  // every lane has read the slot
      if (lane == 0) gen[s] = j + kRedSlots;
    }
  };
  auto one_tile = [&](int j) {
    if constexpr (I8) {
      XFragI8 xf;
      load_xfrag_i8<B1>(xf, xlane8, xs);
      uint32_t acc[CH][4];
      tile_mma_i8<D>(w[j], xf, acc);
      tile_epilogue_i8<D, B1>(sc[j], xf, acc, y);
    } else {
      XFrag<1, XL> xf;
      load_xfrag<1, XL>(xf, xlane, xs);
      float acc[CH][1][4];
      tile_mma<1, XL, D>(w[j], xf, p.shift_mul, acc);
      tile_epilogue<1, XL, D, B1>(sc[j], xf, acc, y);
    }
  };
  for (uint32_t k0 = 0; k0 < total; k0 += R) {
#pragma unroll
    for (int j = 0; j < R; ++j) {
      if (k0 + j < total) {
        one_tile(j);
        if (k0 + j + R < total) load_next(j);  // refill slot j with tile k0 + j + R
        if (ct == te) {
          finish_item(cj);
          ct = ta;
          ++cj;
          xs = xw;
        } else {
          ++ct;
          xs += p.xslot_bytes;
        }
      }
    }
  }
  if (p.g_world > 1) gather_signal(p, G);
}

// --------------------------------------------------------------------------------------
// tcgen05 GEMV (batch <= 8, FP16 activations, uniform depth)
//
// The contraction runs on the 5th-generation tensor cores: per stage of a tile, 8 warps
// decode the int2 codes into FP16 (the code+2 subnormal trick) and store them into tensor
// memory as the A operand (TMEM lane = tile row); one thread issues 8 UMMAs
// (M=128, N=16, K=16 each, kind::f16) whose B operand is the tile column's prepared
// activations in shared memory and whose FP32 accumulators live in tensor memory; warps
// 0..3 read the accumulators back and apply the per-row, per-stage scales.  A producer
// warp streams each tile's stage records plus its activation block into a shared-memory
// ring with 1-D bulk copies (no multicast).
//
// Activation block of one tile column (prep_x_tc_kernel), kTcColBytes:
//   [u = 0..7][n-group 0..1][k-half 0..1][n % 8][8 halves]  UMMA B operand, canonical
//     K-major layout: UMMA u covers lane-quad q = u/2 and word half s = u%2 of the
//     plane record; its k = 2m + t is tile column 32q + 16s + 8t + m, scaled 4^-(m%4)
//   [16 x {2^(24+e), 2^(e+1) * sum}]                     per batch row
//
// TMEM columns: A operand double buffer [0, 128) (64 columns = 128 FP16 per stage),
// accumulators [128, 256): tile parity * 64 + stage * 16.

constexpr uint32_t kTcBBytes = 4096;
constexpr uint32_t kTcColBytes = kTcBBytes + 16 * 8;
constexpr uint32_t kTcThreads = 320;  // warps 0-7 decode (0-3 also epilogue), 8 producer, 9 MMA issuer
constexpr uint32_t kTcTmemCols = 256;
constexpr uint32_t kTcRingBudget = 150 * 1024;

__host__ __device__ inline uint32_t tc_slot_bytes(uint32_t d) {
  return (d * kRecordBytes + kTcColBytes + 127u) / 128u * 128u;
}

// x [batch][cols] FP16 -> per tile column the UMMA B operand + {factor, correction}, the
// same values as prep_x_kernel (tile exponent, rounding, summation order).  Batch rows
// batch..15 are written as zeros.  Grid (C, 16), 128 threads.
__global__ void __launch_bounds__(128) prep_x_tc_kernel(const __half* __restrict__ x, uint32_t cols, uint32_t batch,
                                                        uint8_t* __restrict__ xtc) {
  __shared__ float red[4];
  const uint32_t c = blockIdx.x, b = blockIdx.y, k = threadIdx.x;
  const uint32_t col = c * 128 + k;
  float v = 0.0f;
  if (b < batch && col < cols) v = __half2float(x[static_cast<uint64_t>(b) * cols + col]);
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((k & 31) == 0) red[k >> 5] = a;
  __syncthreads();
  const float amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  int e = 0;
  if (amax > 0.0f) e = max(-100, min(100, ilogbf(amax) - 14));
  const uint32_t m = k & 7, which = (k >> 3) & 3, q = k >> 5, jj = m & 3;
  const float xs = ldexpf(v, -e - 2 * static_cast<int>(jj));
  const __half hi = __float2half_rn(xs);
  const float eff = __half2float(hi);
  const uint32_t u = 2 * q + (which >> 1), kk = 2 * m + (which & 1);
  uint8_t* slot = xtc + static_cast<uint64_t>(c) * kTcColBytes;
  const uint32_t off = u * 512 + (b >> 3) * 256 + (kk >> 3) * 128 + (b & 7) * 16 + (kk & 7) * 2;
  *reinterpret_cast<__half*>(slot + off) = hi;
  float xt = ldexpf(eff, 2 * static_cast<int>(jj));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) xt += __shfl_xor_sync(0xffffffffu, xt, o);
  if ((k & 31) == 0) red[k >> 5] = xt;
  __syncthreads();
  if (k == 0) {
    const float sum = (red[0] + red[1]) + (red[2] + red[3]);
    *reinterpret_cast<float2*>(slot + kTcBBytes + b * 8) = make_float2(ldexpf(1.0f, 24 + e), ldexpf(sum, e + 1));
  }
}

// Bounded mbarrier wait that gives up at once after any earlier timeout of this CTA.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, const GemvParams& p, volatile uint32_t* abort) {
  if (*abort) return false;
  if (mbar_wait(bar, parity, p.error)) return true;
  *abort = 1u;
  return false;
}

template <int D>
__global__ void __launch_bounds__(kTcThreads, 1) gemv_tc_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t S = p.ring_slots, SB = p.slot_stride;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + S * SB);
  uint64_t* empty = full + S;
  uint64_t* a_full = empty + S;   // [2] A buffer written (8 warps)
  uint64_t* a_empty = a_full + 2; // [2] A buffer consumed (MMA commit)
  uint64_t* d_full = a_empty + 2; // [2] tile accumulators ready (MMA commit)
  uint64_t* d_empty = d_full + 2; // [2] tile accumulators read (4 epilogue warps)
  uint32_t* misc = reinterpret_cast<uint32_t*>(d_empty + 2);  // [0] TMEM base, [1] abort, [2] split count, [3..] s_info
  volatile uint32_t* abort = misc + 1;
  const uint64_t total = p.total;
  const uint32_t ctas = static_cast<uint32_t>(total < gridDim.x ? total : gridDim.x), cta = blockIdx.x;
  griddep_launch_dependents();
  if (cta >= ctas) return;
  const uint64_t u0 = unit_start(cta, total, ctas), u1 = unit_start(cta + 1, total, ctas);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t t0 = static_cast<uint32_t>(u0 / D), s0 = static_cast<uint32_t>(u0 % D);
  const uint32_t t_end = static_cast<uint32_t>((u1 - 1) / D), s_end = static_cast<uint32_t>((u1 - 1) % D) + 1;
  const uint32_t ntiles = t_end - t0 + 1;
  constexpr uint32_t kFull = (1u << D) - 1u;
  const uint32_t mask_first = kFull & ~((1u << s0) - 1u), mask_last = (1u << s_end) - 1u;
  auto tile_mask = [&](uint32_t k) {
    return (k == 0 ? mask_first : kFull) & (k == ntiles - 1 ? mask_last : kFull);
  };
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
      mbar_init(&d_full[i], 1);
      mbar_init(&d_empty[i], 4);
    }
    misc[1] = 0u;
    misc[2] = 0u;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&misc[0], kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  SplitRows split{0u, 0u, 0u};

  if (warp == 8) {
    // ---- producer: stage records of tile t0+k and its column's activation block
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
      auto issue = [&](uint32_t k, bool weights, bool acts) {
        const uint32_t slot = k % S, mask = tile_mask(k);
        uint8_t* dst = sm + slot * SB;
        const uint64_t tile = static_cast<uint64_t>(t0) + k;
        if (weights) {
          uint32_t bytes = kTcColBytes;
#pragma unroll
          for (int s = 0; s < D; ++s) bytes += (mask >> s & 1u) ? kRecordBytes : 0u;
          mbar_expect_tx(&full[slot], bytes);
#pragma unroll
          for (int s = 0; s < D; ++s)
            if (mask >> s & 1u) bulk_load(dst + s * kRecordBytes, p.planes[s] + tile * kRecordBytes, kRecordBytes,
                                          &full[slot], pol_w);
        }
        if (acts) {
          const uint32_t c = static_cast<uint32_t>(tile % p.C);
          bulk_load(dst + D * kRecordBytes, p.xfrag + static_cast<uint64_t>(c) * kTcColBytes, kTcColBytes,
                    &full[slot], pol_x);
        }
      };
      const uint32_t first = ntiles < S ? ntiles : S;
      for (uint32_t k = 0; k < first; ++k) issue(k, true, false);  // weights do not depend on earlier kernels
      griddep_wait();
      for (uint32_t k = 0; k < first; ++k) issue(k, false, true);
      for (uint32_t k = first; k < ntiles; ++k) {
        if (!tc_wait(&empty[k % S], ((k / S) - 1) & 1, p, abort)) break;
        issue(k, true, true);
      }
    }
  } else if (warp == 9) {
    // ---- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | ((16u >> 3) << 17) | ((128u >> 4) << 24);  // F32 += F16 x F16, N 16, M 128
      for (uint32_t k = 0; k < ntiles; ++k) {
        const uint32_t slot = k % S, par = k & 1;
        const uint32_t b_addr = smem_u32(sm + slot * SB + D * kRecordBytes);
        bool ok = true;
        for (uint32_t s = 0; s < D && ok; ++s) {
          const uint32_t z = k * D + s, buf = z & 1;
          ok = tc_wait(&a_full[buf], (z >> 1) & 1, p, abort);
          if (ok && s == 0 && k >= 2) ok = tc_wait(&d_empty[par], ((k >> 1) - 1) & 1, p, abort);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (uint32_t u = 0; u < 8; ++u)
            tc_mma_f16_ts(tmem + 128 + par * 64 + s * 16, tmem + buf * 64 + u * 8,
                          umma_desc_kmajor(b_addr + u * 512, 128, 256), idesc, u > 0 ? 1u : 0u);
          tc_commit(&a_empty[buf]);
        }
        if (!ok) break;
        tc_commit(&d_full[par]);
      }
    }
  } else {
    // ---- decode warps 0..7: lane quadrant warp % 4 (tile rows), column half warp / 4
    griddep_wait();  // outputs and partials are written only after earlier kernels complete
    const uint32_t quad = warp & 3, colhalf = warp >> 2;
    const uint32_t rit = quad * 32 + lane;  // tile row of this thread
    const uint32_t rb = rit >> 4, gg = rit & 7, half = (rit >> 3) & 1;
    // this row's four words of its column half: lane quads q = 2*colhalf, +1, words s = 0, 1
    const uint32_t word_off = rb * kRowBlockBytes + (4 * gg + 2 * colhalf) * 16 + half * 4;
    const uint32_t scale_off = rb * kRowBlockBytes + 512 + 4 * gg + 2 * half;
    const uint32_t lane_taddr = tmem + ((quad * 32u) << 16);
    const uint64_t units_per_row = static_cast<uint64_t>(p.C) * D;
    float y[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) y[b] = 0.0f;
    uint32_t row = t0 / p.C, left = p.C - t0 % p.C;

    auto epilogue = [&](uint32_t kk) -> bool {
      const uint32_t par = kk & 1, slot = kk % S, mask = tile_mask(kk);
      if (!tc_wait(&d_full[par], (kk >> 1) & 1, p, abort)) return false;
      tc_fence_after();
      const uint8_t* rec = sm + slot * SB;
      const float2* fg = reinterpret_cast<const float2*>(rec + D * kRecordBytes + kTcBBytes);
#pragma unroll
      for (int s = 0; s < D; ++s) {
        uint32_t acc[8];
        tc_ld_x8(lane_taddr + 128 + par * 64 + s * 16, acc);
        tc_wait_ld();
        const float sigma = (mask >> s & 1u)
                                ? half_bits_to_float(*reinterpret_cast<const uint16_t*>(rec + s * kRecordBytes + scale_off))
                                : 0.0f;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          if (static_cast<uint32_t>(b) < p.batch) {
            const float2 f = fg[b];
            y[b] = fmaf(sigma, fmaf(__uint_as_float(acc[b]), f.x, -f.y), y[b]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&d_empty[par]);
        mbar_arrive(&empty[slot]);
      }
      // end of a tile row for this CTA: store or publish the row's outputs
      if (--left == 0 || kk + 1 == ntiles) {
        const uint64_t rb_u = static_cast<uint64_t>(row) * units_per_row, re_u = rb_u + units_per_row;
        const uint32_t out_row = row * 128 + rit;
        if (rb_u >= u0 && re_u <= u1) {
          if (out_row < p.rows) {
            float bias = 0.0f;
            if (p.bias != nullptr)
              bias = p.bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(p.bias)[out_row])
                                             : static_cast<const float*>(p.bias)[out_row];
#pragma unroll
            for (int b = 0; b < 8; ++b) {
              if (static_cast<uint32_t>(b) >= p.batch) break;
              const uint64_t o = static_cast<uint64_t>(b) * p.rows + out_row;
              if (p.y_dtype == HQB_F16) static_cast<__half*>(p.y)[o] = __float2half_rn(y[b] + bias);
              else static_cast<float*>(p.y)[o] = y[b] + bias;
            }
          }
        } else {
          float* part = p.partials + static_cast<uint64_t>(cta * 2 + (rb_u <= u0 ? 0u : 1u)) * p.batch * 128;
#pragma unroll
          for (int b = 0; b < 8; ++b)
            if (static_cast<uint32_t>(b) < p.batch) part[b * 128 + rit] = y[b];
          if (split.count == 0) split.row0 = row;
          else split.row1 = row;
          ++split.count;
        }
#pragma unroll
        for (int b = 0; b < 8; ++b) y[b] = 0.0f;
        ++row;
        left = p.C;
      }
      return true;
    };

    bool ok = true;
    for (uint32_t k = 0; k < ntiles && ok; ++k) {
      const uint32_t slot = k % S;
      ok = tc_wait(&full[slot], (k / S) & 1, p, abort);
      const uint8_t* rec = sm + slot * SB;
      for (uint32_t s = 0; s < D && ok; ++s) {
        const uint32_t z = k * D + s, buf = z & 1;
        if (z >= 2) ok = tc_wait(&a_empty[buf], ((z >> 1) - 1) & 1, p, abort);
        if (!ok) break;
        const uint8_t* r = rec + s * kRecordBytes + word_off;
        const uint32_t w[4] = {lds32(r), lds32(r + 8), lds32(r + 16), lds32(r + 24)};
        uint32_t a[32];
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
          const uint32_t h = __umulhi(w[wi], p.shift_mul);
#pragma unroll
          for (int m = 0; m < 8; ++m) a[wi * 8 + m] = int2_pair(w[wi], h, m);
        }
        tc_st_x32(lane_taddr + buf * 64 + colhalf * 32, a);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[buf]);
      }
      if (ok && colhalf == 0 && k >= 1) ok = epilogue(k - 1);
    }
    if (ok && colhalf == 0 && ntiles >= 1) ok = epilogue(ntiles - 1);
    if (threadIdx.x == 0) {
      misc[2] = split.count;
      misc[12] = split.row0;
      misc[13] = split.row1;
    }
  }
  tc_fence_before();
  __syncthreads();
  // split tile rows: thread 0 holds this CTA's list (a CTA-uniform decision)
  const uint32_t nsplit = misc[2];
  if (nsplit != 0 && *abort == 0u) {
    SplitRows sp{misc[12], misc[13], nsplit};
    finish_split_rows<1>(p, sp, static_cast<uint64_t>(p.C) * D, total, ctas, misc + 3, kTcThreads);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, kTcTmemCols);
}

// Waits (one thread, bounded) until every rank's counter in `flags` reached *epoch + 1,
// then advances the epoch.
__global__ void gather_wait_kernel(const uint32_t* flags, uint32_t world, uint32_t* epoch, int* device_flags,
                                   unsigned long long limit_ns) {
  if (threadIdx.x != 0) return;
  const uint32_t target = *epoch + 1u;
  const unsigned long long start = global_timer_ns();
  for (uint32_t r = 0; r < world; ++r) {
    while (static_cast<int32_t>(ld_acquire_sys(flags + r) - target) < 0) {
      if (global_timer_ns() - start > limit_ns) {
        if (device_flags != nullptr) atomicOr(device_flags, HQB_DEVERR_TIMEOUT);
        *epoch = target;
        return;
      }
    }
  }
  *epoch = target;
}

// Split tile rows: the parts of the contributing CTAs, summed in CTA order, plus
// bias.  Launched as a programmatic dependent of the GEMV; griddepcontrol.wait makes
// the GEMV's stores visible.  One block per tile row; whole rows exit at once.
__global__ void __launch_bounds__(256) fixup_kernel(const __grid_constant__ GemvParams p, uint32_t grid) {
  griddep_wait();
  griddep_launch_dependents();
  const uint64_t total = p.plan != nullptr ? static_cast<uint64_t>(p.plan[p.R]) : p.total;
  const uint32_t ctas = static_cast<uint32_t>(total < grid ? total : grid);
  const uint32_t r = blockIdx.x;
  if (r >= p.R || total == 0) return;
  const RowSplit rs = row_split(p, r, total, ctas);
  if (rs.first == rs.last) return;
  // CTA rs.first holds the row in its second slot when its range began in an earlier
  // row; every later contributor starts inside this row (first slot).
  const uint64_t per_row = static_cast<uint64_t>(p.C) * p.prefix;
  const uint64_t rb = row_begin(r, p.plan, per_row);
  const uint32_t first_slot = unit_start(rs.first, total, ctas) < rb ? 1u : 0u;
  const uint64_t cta_stride = 2ull * p.batch * 128;
  for (uint32_t e = threadIdx.x; e < p.batch * 128; e += blockDim.x) {
    const uint32_t b = e >> 7, rit = e & 127;
    const uint32_t row = r * 128 + rit;
    if (row >= p.rows) continue;
    const float* src = p.partials + static_cast<uint64_t>(b) * 128 + rit;
    float sum = 0.0f;
    sum += src[rs.first * cta_stride + first_slot * p.batch * 128];
    uint32_t i = rs.first + 1;
    for (; i + 4 <= rs.last + 1; i += 4) {
      const float v0 = src[i * cta_stride], v1 = src[(i + 1) * cta_stride];
      const float v2 = src[(i + 2) * cta_stride], v3 = src[(i + 3) * cta_stride];
      sum += v0;
      sum += v1;
      sum += v2;
      sum += v3;
    }
    for (; i <= rs.last; ++i) sum += src[i * cta_stride];
    // the partials region is zero between launches
    const_cast<float*>(src)[rs.first * cta_stride + first_slot * p.batch * 128] = 0.0f;
    for (i = rs.first + 1; i <= rs.last; ++i) const_cast<float*>(src)[i * cta_stride] = 0.0f;
    if (p.bias != nullptr)
      sum += p.bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(p.bias)[row])
                                     : static_cast<const float*>(p.bias)[row];
    const uint64_t o = static_cast<uint64_t>(b) * p.rows + row;
    if (p.y_dtype == HQB_F16) static_cast<__half*>(p.y)[o] = __float2half_rn(sum);
    else static_cast<float*>(p.y)[o] = sum;
  }
}

// --------------------------------------------------------------------------------------
// decode (bit-exact dense weights), depth plan, prefix-0 fill

__global__ void __launch_bounds__(256) decode_kernel(hqb_plane_matrix m, uint32_t prefix,
                                                     const uint8_t* __restrict__ depth, float* __restrict__ out) {
  const uint32_t tile = blockIdx.x;
  const uint32_t r = tile / m.grid_cols, c = tile % m.grid_cols;
  const uint32_t rb = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  uint32_t d = prefix;
  if (depth != nullptr) d = clamp_depth(depth[tile], m.stage_count);
  uint32_t words[HQB_MAX_STAGES][4];
  float sc[HQB_MAX_STAGES][2];
#pragma unroll
  for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) {
    if (s < d) {
      const uint8_t* rec = static_cast<const uint8_t*>(m.planes[s]) + static_cast<uint64_t>(tile) * kRecordBytes +
                           rb * kRowBlockBytes;
      const uint4 w = *reinterpret_cast<const uint4*>(rec + lane * 16);
      words[s][0] = w.x;
      words[s][1] = w.y;
      words[s][2] = w.z;
      words[s][3] = w.w;
      const uint32_t pair = *reinterpret_cast<const uint32_t*>(rec + 512 + g * 4);
      sc[s][0] = half_bits_to_float(pair & 0xFFFFu);
      sc[s][1] = half_bits_to_float(pair >> 16);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t row = static_cast<uint64_t>(r) * 128 + rb * 16 + g + 8 * (i & 1);
    const uint64_t col0 = static_cast<uint64_t>(c) * 128 + 32 * q + 16 * (i >> 1);
    if (row >= m.rows) continue;
#pragma unroll 4
    for (int k = 0; k < 16; ++k) {
      if (col0 + k >= m.cols) break;
      float wsum = 0.0f;
#pragma unroll
      for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) {
        if (s >= d) break;
        const float code = static_cast<float>(static_cast<int>((words[s][i] >> (2 * k)) & 3u) - 2);
        wsum = __fadd_rn(wsum, __fmul_rn(code, sc[s][i & 1]));
      }
      out[row * m.cols + col0 + k] = wsum;
    }
  }
}

__global__ void __launch_bounds__(1024) depth_plan_kernel(const uint8_t* __restrict__ depth, uint32_t R,
                                                          uint32_t C, uint32_t stage_count,
                                                          uint32_t* __restrict__ plan, int* flags) {
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (uint32_t r = warp; r < R; r += nw) {
    uint32_t cost = 0;
    int bad = 0;
    for (uint32_t c = lane; c < C; c += 32) {
      const uint32_t d = depth[static_cast<uint64_t>(r) * C + c];
      if (d < 1 || d > stage_count) bad = 1;
      cost += clamp_depth(d, stage_count);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      cost += __shfl_xor_sync(0xffffffffu, cost, o);
      bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (lane == 0) {
      plan[r + 1] = cost;
      if (bad && flags != nullptr) atomicOr(flags, HQB_DEVERR_DEPTH);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    plan[0] = 0;
    for (uint32_t r = 0; r < R; ++r) {
      run += plan[r + 1];
      plan[r + 1] = run;
    }
  }
}

__global__ void fill_kernel(const void* bias, int bias_dtype, void* y, int y_dtype, uint32_t rows, uint32_t batch) {
  const uint64_t n = static_cast<uint64_t>(rows) * batch;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t row = static_cast<uint32_t>(i % rows);
    float v = 0.0f;
    if (bias != nullptr)
      v = bias_dtype == HQB_F16 ? __half2float(static_cast<const __half*>(bias)[row]) : static_cast<const float*>(bias)[row];
    if (y_dtype == HQB_F16) static_cast<__half*>(y)[i] = __float2half_rn(v);
    else static_cast<float*>(y)[i] = v;
  }
}

// --------------------------------------------------------------------------------------
// host side

int device_sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cache[device] = v;
  }
  return cache[device];
}

namespace {

struct WsLayout {
  uint64_t counters, partials, xfrag, xtc, total;
};

// [error word][split-row counters: R uint32][split-row partials: G x 2 x batch x 128
// FP32, or G x batch x 128 flagged 64-bit words for the uniform stream-K kernel]
// [prepared activations: mma fragments][prepared activations: tcgen05 B blocks].  The
// error word, the counters and the partials must start at zero (hqb_workspace_init);
// counters and partials return to zero at the end of every launch.
WsLayout ws_layout(uint32_t R, uint32_t C, uint32_t batch, uint32_t xl, int sms) {
  WsLayout L{};
  L.counters = 256;
  L.partials = L.counters + round_up((static_cast<uint64_t>(R) + 1) * 4, 256);  // + launch-done counter
  const uint64_t gmax = static_cast<uint64_t>(sms) * kMaxCtasPerSm;
  L.xfrag = L.partials + round_up(gmax * 2 * batch * 128 * 4, 256);
  const uint32_t xslot = std::max(xslot_bytes_for(batch, xl), batch <= 2 ? xslot_i8_bytes(batch) : 0u);
  L.xtc = L.xfrag + round_up(static_cast<uint64_t>(C) * xslot, 256);
  L.total = L.xtc + round_up(static_cast<uint64_t>(C) * kTcColBytes, 256);
  return L;
}

bool plane_matrix_ok(const hqb_plane_matrix* m) {
  if (m == nullptr || m->rows == 0 || m->cols == 0 || m->stage_count == 0 || m->stage_count > HQB_MAX_STAGES)
    return false;
  if (m->grid_rows != (m->rows + 127) / 128 || m->grid_cols != (m->cols + 127) / 128) return false;
  if (m->rows > 0xFFFFFFFFull || m->cols > 0xFFFFFFFFull) return false;
  return true;
}

bool stage_planes_ok(const hqb_plane_matrix* m, uint32_t needed) {
  for (uint32_t s = 0; s < needed; ++s) {
    if (m->planes[s] == nullptr || (reinterpret_cast<uintptr_t>(m->planes[s]) & 15u) != 0) return false;
  }
  return true;
}


template <int NB, int XL, bool B1 = false>
GemvKernel pick_uniform_depth(uint32_t d) {
  switch (d) {
    case 1: return gemv_uniform_kernel<NB, XL, 1, B1>;
    case 2: return gemv_uniform_kernel<NB, XL, 2, B1>;
    case 3: return gemv_uniform_kernel<NB, XL, 3, B1>;
    default: return gemv_uniform_kernel<NB, XL, 4, B1>;
  }
}

template <int XL, bool B1>
GemvKernel pick_uniform_i8(uint32_t d) {
  switch (d) {
    case 1: return gemv_uniform_kernel<1, XL, 1, B1, true>;
    case 2: return gemv_uniform_kernel<1, XL, 2, B1, true>;
    case 3: return gemv_uniform_kernel<1, XL, 3, B1, true>;
    default: return gemv_uniform_kernel<1, XL, 4, B1, true>;
  }
}

GemvKernel pick_mixed_i8(uint32_t batch, uint32_t xl) {
  if (xl == 1) return batch == 1 ? gemv_unit_kernel<1, true> : gemv_unit_kernel<1, false>;
  return batch == 1 ? gemv_unit_kernel<2, true> : gemv_unit_kernel<2, false>;
}

GemvKernel pick_uniform_kernel(uint32_t nb, uint32_t xl, uint32_t d, uint32_t batch, bool i8) {
  if (i8 && xl == 1) return batch == 1 ? pick_uniform_i8<1, true>(d) : pick_uniform_i8<1, false>(d);
  if (i8) return batch == 1 ? pick_uniform_i8<2, true>(d) : pick_uniform_i8<2, false>(d);
  if (nb == 1 && xl == 1 && batch == 1) return pick_uniform_depth<1, 1, true>(d);
  if (nb == 1) return xl == 1 ? pick_uniform_depth<1, 1>(d) : pick_uniform_depth<1, 2>(d);
  return xl == 1 ? pick_uniform_depth<2, 1>(d) : pick_uniform_depth<2, 2>(d);
}

template <int XL, bool B1, bool I8 = false>
GemvKernel pick_rows_depth(uint32_t d) {
  switch (d) {
    case 1: return gemv_rows_kernel<XL, 1, B1, I8>;
    case 2: return gemv_rows_kernel<XL, 2, B1, I8>;
    case 3: return gemv_rows_kernel<XL, 3, B1, I8>;
    default: return gemv_rows_kernel<XL, 4, B1, I8>;
  }
}

GemvKernel pick_rows_kernel(uint32_t xl, uint32_t d, uint32_t batch, bool i8) {
  if (i8 && xl == 1) return batch == 1 ? pick_rows_depth<1, true, true>(d) : pick_rows_depth<1, false, true>(d);
  if (i8) return batch == 1 ? pick_rows_depth<2, true, true>(d) : pick_rows_depth<2, false, true>(d);
  if (xl == 1) return batch == 1 ? pick_rows_depth<1, true>(d) : pick_rows_depth<1, false>(d);
  return pick_rows_depth<2, false>(d);
}

// Fragment bytes per warp area of the row-block kernel: the most tile columns any warp's
// unit range touches, times the slot size.
uint32_t rows_xw_bytes(uint32_t C, uint32_t d, uint32_t xslot) {
  const uint32_t U = C * d;
  uint32_t nt = 0;
  for (uint32_t w = 0; w < kRowsWarps; ++w) {
    const uint32_t ua = rows_unit_start(w, U), ub = rows_unit_start(w + 1, U);
    if (ua < ub) nt = std::max(nt, (ub - 1) / d - ua / d + 1);
  }
  return nt * xslot;
}

GemvKernel pick_stream_kernel(uint32_t nb, uint32_t xl) {
  if (nb == 1) return xl == 1 ? gemv_stream_kernel<1, 1> : gemv_stream_kernel<1, 2>;
  return xl == 1 ? gemv_stream_kernel<2, 1> : gemv_stream_kernel<2, 2>;
}

GemvKernel pick_kernel(uint32_t nb, uint32_t xl, bool simt) {
  if (simt) return gemv_kernel<1, 1, true>;
  if (nb == 1) return xl == 1 ? gemv_kernel<1, 1, false> : gemv_kernel<1, 2, false>;
  return xl == 1 ? gemv_kernel<2, 1, false> : gemv_kernel<2, 2, false>;
}

struct RingShape {
  uint32_t slots, stride, smem;
};

// Ring geometry: a slot holds one run of up to `cap` stages of a tile; enough slots to
// keep about kUnitsInFlight tile-stages in flight within the shared-memory budget.
// slot_x: activation bytes per slot (0 when the whole activation set is resident);
// resident: bytes of that set.
RingShape ring_shape(uint32_t slot_x, uint32_t cap, uint32_t resident) {
  RingShape r{};
  r.stride = static_cast<uint32_t>(round_up(kHdrBytes + slot_x + cap * kRecordBytes, 16));
  r.slots = std::max<uint32_t>(2, std::min<uint32_t>(std::max<uint32_t>(1, kUnitsInFlight / cap), kSmemBudget / r.stride));
  r.smem = r.slots * r.stride + resident + (2 * r.slots + 1) * 8;
  return r;
}

constexpr uint32_t kXResidentMax = 64 * 1024;
// int8 limb slots a stream-K CTA holds (min(C, its tiles) of them): two CTAs per SM up
// to 104 KB each; more use the FP16-fragment kernels.
constexpr uint32_t kXResidentMaxI8 = 104 * 1024;
constexpr uint64_t kFusedTilesMax = 24;

uint32_t gemv_smem_cap() {
  uint32_t m = 0;
  for (uint32_t cap = 1; cap <= HQB_MAX_STAGES; ++cap)
    m = std::max(m, ring_shape(xslot_bytes_for(HQB_MAX_BATCH, 2), cap, 0).smem);
  for (uint32_t cap = 1; cap <= HQB_MAX_STAGES; ++cap)
    m = std::max(m, ring_shape(0, cap, kXResidentMax).smem);
  return std::max(std::max(std::max(m, kSmemBudget + 1024), kRowsSmemMax), kXResidentMaxI8 + 4096 + 256);
}

// Resident CTAs per SM for a kernel variant at a given shared-memory size (cached).
int ctas_per_sm(GemvKernel k, uint32_t smem, int device, uint32_t threads) {
  struct Entry {
    GemvKernel k;
    uint32_t smem;
    int device;
    int ctas;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].k == k && cache[i].smem == smem && cache[i].device == device) return cache[i].ctas;
  // The attribute is a per-kernel maximum: set it once to the largest size any batch
  // needs, so a later smaller request can never lower it below a cached larger one.
  const uint32_t smem_cap = gemv_smem_cap();
  if (cudaFuncSetAttribute(reinterpret_cast<const void*>(k), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem_cap)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, static_cast<int>(threads), smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  n = std::min<int>(n, kMaxCtasPerSm);
  if (used < 64) cache[used++] = Entry{k, smem, device, n};
  return n;
}

template <int D>
cudaError_t launch_tc(const GemvParams& p, uint32_t grid, uint32_t smem, bool pdl, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_status = cudaSuccess;
  std::call_once(once, [] {
    attr_status = cudaFuncSetAttribute(gemv_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (attr_status != cudaSuccess) return attr_status;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (pdl) {
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gemv_tc_kernel<D>, p);
}

// Raw activation rows that load as aligned vectors: a 16-byte aligned start and rows of
// a multiple of 16 bytes.
bool x_rows_vec(const void* x, uint64_t cols, uint32_t xl) {
  return (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (cols * (xl == 1 ? 2 : 4)) % 16 == 0;
}

cudaError_t launch_prep(const void* x, int x_dtype, uint64_t cols, uint32_t batch, void* xfrag, cudaStream_t st) {
  const uint32_t C = static_cast<uint32_t>((cols + 127) / 128);
  const uint32_t xl = x_dtype == HQB_F32 ? 2 : 1;
  const uint32_t blocks = (C * batch + 3) / 4;  // one warp per (tile column, batch row)
  const uint32_t xs = xslot_bytes_for(batch, xl);
  const uint32_t vec = x_rows_vec(x, cols, xl) ? 1u : 0u;
  if (x_dtype == HQB_F32)
    prep_x_kernel<2, float><<<blocks, 128, 0, st>>>(static_cast<const float*>(x), static_cast<uint32_t>(cols), batch,
                                                    C, static_cast<uint8_t*>(xfrag), xs, vec);
  else
    prep_x_kernel<1, __half><<<blocks, 128, 0, st>>>(static_cast<const __half*>(x), static_cast<uint32_t>(cols),
                                                     batch, C, static_cast<uint8_t*>(xfrag), xs, vec);
  return cudaGetLastError();
}

}  // namespace
}  // namespace hqb

using namespace hqb;

extern "C" {

HQB_API int hqb_version(void) { return 1; }

HQB_API const char* hqb_status_string(int status) {
  switch (status) {
    case HQB_OK: return "success";
    case HQB_ERR_INVALID: return "invalid argument (nothing enqueued)";
    case HQB_ERR_UNSUPPORTED: return "geometry not supported by the plane layout";
    case HQB_ERR_SCRATCH_LIMIT: return "work needs more scratch than HQB_NOALLOC_SCRATCH_BYTES (nothing enqueued)";
    default: return cudaGetErrorString(static_cast<cudaError_t>(status));
  }
}

HQB_API uint64_t hqb_plane_bytes(const hqb_geometry* g) {
  if (g == nullptr || g->tile_rows != HQB_TILE || g->tile_columns != HQB_TILE || g->group_size != HQB_TILE) return 0;
  if (g->original_rows == 0 || g->original_columns == 0) return 0;
  const uint64_t R = (g->original_rows + 127) / 128, C = (g->original_columns + 127) / 128;
  if (g->padded_rows != R * 128 || g->padded_columns != C * 128) return 0;
  uint64_t tiles = 0, bytes = 0;
  if (!mul_ok(R, C, &tiles) || !mul_ok(tiles, kRecordBytes, &bytes)) return 0;
  return bytes;
}

HQB_API int hqb_repack_stage(const hqb_geometry* g, const hqb_raw_stage* stage, void* plane, int* device_flags,
                             void* stream) {
  const uint64_t bytes = hqb_plane_bytes(g);
  if (g != nullptr && bytes == 0 &&
      (g->tile_rows != HQB_TILE || g->tile_columns != HQB_TILE || g->group_size != HQB_TILE))
    return HQB_ERR_UNSUPPORTED;
  if (bytes == 0 || stage == nullptr || plane == nullptr || stage->packed_codes == nullptr ||
      stage->scale_fp16_bits == nullptr || (reinterpret_cast<uintptr_t>(plane) & 15u) != 0)
    return HQB_ERR_INVALID;
  const uint64_t R = g->padded_rows / 128, C = g->padded_columns / 128;
  if (g->original_rows > 0xFFFFFFFFull || g->original_columns > 0xFFFFFFFFull || R * C > 0x7FFFFFFFull)
    return HQB_ERR_INVALID;
  if (stage->packed_code_bytes != g->padded_rows * g->padded_columns / 4 || stage->scale_count != R * C * 128)
    return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  const int aligned4 = (reinterpret_cast<uintptr_t>(stage->packed_codes) & 3u) == 0;
  repack_kernel<<<static_cast<unsigned>(R * C), 256, 0, as_stream(stream)>>>(
      stage->packed_codes, stage->scale_fp16_bits, static_cast<uint8_t*>(plane), g->padded_columns / 4,
      static_cast<uint32_t>(g->original_rows), static_cast<uint32_t>(g->original_columns), static_cast<uint32_t>(C),
      device_flags, aligned4);
  return cudaGetLastError();
}

HQB_API uint64_t hqb_xfrag_bytes(uint64_t cols, uint32_t batch, int x_dtype) {
  if (cols == 0 || batch == 0 || batch > HQB_MAX_BATCH || (x_dtype != HQB_F16 && x_dtype != HQB_F32)) return 0;
  return ((cols + 127) / 128) * xslot_bytes_for(batch, x_dtype == HQB_F32 ? 2 : 1);
}

HQB_API int hqb_prepare_x(const void* x, int x_dtype, uint64_t cols, uint32_t batch, void* xfrag, void* stream) {
  if (x == nullptr || xfrag == nullptr || hqb_xfrag_bytes(cols, batch, x_dtype) == 0 || cols > 0xFFFFFFFFull ||
      (reinterpret_cast<uintptr_t>(xfrag) & 15u) != 0)
    return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  return launch_prep(x, x_dtype, cols, batch, xfrag, as_stream(stream));
}

HQB_API uint64_t hqb_workspace_bytes(const hqb_plane_matrix* m, uint32_t batch, int x_dtype, int device) {
  if (!plane_matrix_ok(m) || batch == 0 || batch > HQB_MAX_BATCH || (x_dtype != HQB_F16 && x_dtype != HQB_F32))
    return 0;
  const int sms = device_sm_count(device);
  if (sms <= 0) return 0;
  return ws_layout(m->grid_rows, m->grid_cols, batch, x_dtype == HQB_F32 ? 2 : 1, sms).total;
}

HQB_API int hqb_workspace_init(void* workspace, uint64_t bytes, void* stream) {
  if (workspace == nullptr || bytes < 256) return HQB_ERR_INVALID;
  return cudaMemsetAsync(workspace, 0, bytes, as_stream(stream));
}

HQB_API int hqb_workspace_error(const void* workspace, int* host_flags, void* stream) {
  if (workspace == nullptr || host_flags == nullptr) return HQB_ERR_INVALID;
  cudaError_t e = cudaMemcpyAsync(host_flags, workspace, sizeof(int), cudaMemcpyDeviceToHost, as_stream(stream));
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(as_stream(stream));
}

HQB_API uint64_t hqb_depth_plan_bytes(uint32_t grid_rows) { return (static_cast<uint64_t>(grid_rows) + 1) * 4; }

HQB_API int hqb_depth_plan(const uint8_t* depth, uint32_t grid_rows, uint32_t grid_cols, uint32_t stage_count,
                           uint32_t* plan, int* device_flags, void* stream) {
  if (depth == nullptr || plan == nullptr || grid_rows == 0 || grid_cols == 0 || stage_count == 0 ||
      stage_count > HQB_MAX_STAGES || static_cast<uint64_t>(grid_rows) * grid_cols * HQB_MAX_STAGES > 0xFFFFFFFFull)
    return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  depth_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(depth, grid_rows, grid_cols, stage_count, plan, device_flags);
  return cudaGetLastError();
}

}  // extern "C"

namespace {

// hqb_gemv_ex, optionally with the fused all-gather of the outputs (gather != nullptr).
int gemv_impl(const hqb_plane_matrix* m, uint32_t prefix, const uint8_t* depth, const uint32_t* depth_plan,
              const void* x, int x_dtype, uint32_t batch, int x_prepared, const void* bias, int bias_dtype, void* y,
              int y_dtype, void* workspace, uint64_t workspace_bytes, uint32_t flags, void* stream,
              const hqb_gather* gather, hqb_launch_info* info = nullptr) {
  // info != nullptr: a dry run (hqb_gemv_query) -- the same validation and choices, the
  // launches described in *info instead of enqueued
  auto describe = [&](const char* kernel, uint32_t launches, bool i8, uint64_t grid, uint32_t block,
                      uint32_t smem) -> int {
    *info = hqb_launch_info{};
    info->launches = launches;
    info->int8_limbs = i8 ? 1u : 0u;
    info->grid = static_cast<uint32_t>(grid);
    info->block = block;
    info->smem_bytes = smem;
    std::strncpy(info->kernel, kernel, sizeof(info->kernel) - 1);
    return HQB_OK;
  };
  if (!plane_matrix_ok(m) || x == nullptr || (y == nullptr && gather == nullptr) || workspace == nullptr)
    return HQB_ERR_INVALID;
  if (gather != nullptr) {
    if (gather->world < 2 || gather->world > HQB_MAX_PEERS || gather->rank >= gather->world ||
        gather->slot_rows < m->rows || depth != nullptr || prefix == 0)
      return HQB_ERR_INVALID;
    for (uint32_t r = 0; r < gather->world; ++r)
      if (gather->peer_y[r] == nullptr || gather->peer_flags[r] == nullptr) return HQB_ERR_INVALID;
    if (flags & (HQB_FLAG_SIMT | HQB_FLAG_RING | HQB_FLAG_TCGEN05)) return HQB_ERR_UNSUPPORTED;
  }
  if (batch == 0 || batch > HQB_MAX_BATCH) return HQB_ERR_INVALID;
  if ((x_dtype != HQB_F16 && x_dtype != HQB_F32) || (y_dtype != HQB_F16 && y_dtype != HQB_F32)) return HQB_ERR_INVALID;
  if (bias != nullptr && bias_dtype != HQB_F16 && bias_dtype != HQB_F32) return HQB_ERR_INVALID;
  if ((depth == nullptr) != (depth_plan == nullptr)) return HQB_ERR_INVALID;
  if ((flags & HQB_FLAG_STREAMK) && (flags & HQB_FLAG_ROWBLOCK)) return HQB_ERR_INVALID;
  const bool mixed = depth != nullptr;
  if (!mixed && prefix > m->stage_count) return HQB_ERR_INVALID;
  const bool simt = (flags & HQB_FLAG_SIMT) != 0;
  if (simt && (batch > 8 || x_dtype != HQB_F16)) return HQB_ERR_INVALID;
  if (!stage_planes_ok(m, mixed ? m->stage_count : prefix)) return HQB_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return HQB_ERR_INVALID;
  if (x_prepared && (reinterpret_cast<uintptr_t>(x) & 15u) != 0) return HQB_ERR_INVALID;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  const int sms = device_sm_count(device);
  if (sms <= 0) return cudaErrorNoDevice;
  const uint32_t xl = x_dtype == HQB_F32 ? 2 : 1;
  const WsLayout L = ws_layout(m->grid_rows, m->grid_cols, batch, xl, sms);
  if (workspace_bytes < L.total) return HQB_ERR_INVALID;
  if (info == nullptr) {
    const cudaError_t prior = take_prior_error();
    if (prior != cudaSuccess) return prior;
  }
  const cudaStream_t st = as_stream(stream);
  if (!mixed && prefix == 0) {
    if (info) return describe("fill_kernel", 1, false, std::min<uint64_t>((m->rows * batch + 255) / 256, 4096), 256, 0);
    const uint64_t n = m->rows * batch;
    const unsigned blocks = static_cast<unsigned>(std::min<uint64_t>((n + 255) / 256, 4096));
    fill_kernel<<<blocks, 256, 0, st>>>(bias, bias_dtype, y, y_dtype, static_cast<uint32_t>(m->rows), batch);
    return cudaGetLastError();
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  // tcgen05 comparison path (on request): uniform depth, raw FP16 activations, batch <= 8
  if ((flags & HQB_FLAG_TCGEN05) && gather == nullptr && !mixed && !simt && !x_prepared && x_dtype == HQB_F16 &&
      batch <= 8 && !(flags & HQB_FLAG_RING)) {
    const uint32_t C = m->grid_cols;
    if (info) {
      const uint32_t sb = tc_slot_bytes(prefix);
      const uint32_t slots = std::max<uint32_t>(3, std::min<uint32_t>(16, kTcRingBudget / sb));
      const uint64_t total = static_cast<uint64_t>(m->grid_rows) * C * prefix;
      return describe("gemv_tc_kernel", 2, false, std::min<uint64_t>(sms, total), kTcThreads,
                      slots * sb + (2 * slots + 8) * 8 + 16 * 4);
    }
    prep_x_tc_kernel<<<dim3(C, 16), 128, 0, st>>>(static_cast<const __half*>(x), static_cast<uint32_t>(m->cols), batch,
                                                  ws + L.xtc);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    GemvParams p{};
    for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) p.planes[s] = static_cast<const uint8_t*>(m->planes[s]);
    p.xfrag = ws + L.xtc;
    p.bias = bias;
    p.y = y;
    p.error = reinterpret_cast<int*>(ws);
    p.partials = reinterpret_cast<float*>(ws + L.partials);
    p.counters = reinterpret_cast<uint32_t*>(ws + L.counters);
    p.rows = static_cast<uint32_t>(m->rows);
    p.R = m->grid_rows;
    p.C = C;
    p.prefix = prefix;
    p.stage_count = m->stage_count;
    p.batch = batch;
    p.bias_dtype = bias_dtype;
    p.y_dtype = y_dtype;
    p.cols = static_cast<uint32_t>(m->cols);
    p.shift_mul = 1u << 24;
    p.total = static_cast<uint64_t>(m->grid_rows) * C * prefix;
    const uint32_t sb = tc_slot_bytes(prefix);
    const uint32_t slots = std::max<uint32_t>(3, std::min<uint32_t>(16, kTcRingBudget / sb));
    p.ring_slots = slots;
    p.slot_stride = sb;
    const uint32_t smem = slots * sb + (2 * slots + 8) * 8 + 16 * 4;
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(static_cast<uint64_t>(sms), p.total));
    const bool pdl = (flags & HQB_FLAG_PDL) != 0;
    switch (prefix) {
      case 1: e = launch_tc<1>(p, grid, smem, pdl, st); break;
      case 2: e = launch_tc<2>(p, grid, smem, pdl, st); break;
      case 3: e = launch_tc<3>(p, grid, smem, pdl, st); break;
      default: e = launch_tc<4>(p, grid, smem, pdl, st); break;
    }
    if (e != cudaSuccess) {
      cudaGetLastError();
      return e;
    }
    return cudaGetLastError();
  }
  // Bulk-copy kernel (hqb_bulk.cu): raw FP16 or FP32 x at batch <= 2, uniform prefix or a
  // depth map -- the default there.  Plane bytes reach shared memory through large 1-D
  // bulk copies issued ahead of griddepcontrol.wait; activations become int8 limbs.
  // Default for wide layers (>= 128 tile columns, i.e. K >= 16384) of >= 96 MB of selected
  // planes at prefix >= 2, where its streaming rate wins (8192x28672 at prefix 3: 35.0 us
  // against 39.2 us); elsewhere the register-ring kernels keep the lower fixed cost per
  // launch (B200 timings of both).  HQB_FLAG_BULK forces it.
  const bool bulk_form = !simt && !x_prepared && batch <= 2 &&
                         !(flags & (HQB_FLAG_RING | HQB_FLAG_F16MMA | HQB_FLAG_STREAMK | HQB_FLAG_ROWBLOCK));
  const uint64_t sel_plane_bytes = static_cast<uint64_t>(m->grid_rows) * m->grid_cols * kRecordBytes * prefix;
  // FP32 activations with a depth map take it too: its limbs keep activations of 2^100 and
  // more exact (the register-ring depth-map kernel gives NaN rows for them).
  const bool bulk_default = (mixed && x_dtype == HQB_F32) ||
                            (!mixed && prefix >= 2 && m->grid_cols >= 128 && sel_plane_bytes >= (96ull << 20));
  if (bulk_form && ((flags & HQB_FLAG_BULK) || bulk_default)) {
    const uint32_t kd = mixed ? HQB_MAX_STAGES : prefix;
    // units: exact for a uniform prefix; a depth map's total lives on the device, so the
    // launch is sized for the largest (every tile at stage_count)
    const uint64_t tiles = static_cast<uint64_t>(m->grid_rows) * m->grid_cols;
    const uint64_t units = tiles * (mixed ? m->stage_count : prefix);
    const uint32_t xs8 = xslot_i8_bytes(batch);
    const BulkPlan bp = bulk_plan(tiles, mixed ? m->stage_count : prefix, mixed, m->grid_cols, xs8, sms);
    if (bp.smem <= bulk_smem_max()) {
      // limbs: built per CTA from raw x, or one preparation launch shared by all CTAs when
      // CTAs touch many tile columns
      const bool prep = bp.res_slots > kFusedTilesMax;
      if (info) return describe("gemv_bulk_kernel", prep ? 2u : 1u, true, bp.grid, 288, bp.smem);
      GemvParams p{};
      for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) p.planes[s] = static_cast<const uint8_t*>(m->planes[s]);
      p.depth = depth;
      p.plan = depth_plan;
      p.bias = bias;
      p.y = y;
      p.error = reinterpret_cast<int*>(ws);
      p.partials = reinterpret_cast<float*>(ws + L.partials);
      p.counters = reinterpret_cast<uint32_t*>(ws + L.counters);
      p.rows = static_cast<uint32_t>(m->rows);
      p.R = m->grid_rows;
      p.C = m->grid_cols;
      p.prefix = mixed ? 0 : prefix;
      p.stage_count = m->stage_count;
      p.batch = batch;
      p.xslot_bytes = xs8;
      p.bias_dtype = bias_dtype;
      p.y_dtype = y_dtype;
      p.cols = static_cast<uint32_t>(m->cols);
      p.pdl = (flags & HQB_FLAG_PDL) ? 1u : 0u;
      p.total = mixed ? 0 : units;
      if (gather != nullptr) {
        p.g_world = gather->world;
        p.g_rank = gather->rank;
        p.g_slot_rows = gather->slot_rows;
        for (uint32_t r = 0; r < gather->world; ++r) {
          p.g_peer_y[r] = gather->peer_y[r];
          p.g_peer_flags[r] = gather->peer_flags[r];
        }
        p.g_done = reinterpret_cast<uint32_t*>(ws + L.counters) + m->grid_rows;
      }
      if (prep) {
        e = launch_prep_limbs(x, x_dtype, m->cols, batch, ws + L.xfrag, (flags & HQB_FLAG_PDL) != 0, st);
        if (e != cudaSuccess) {
          cudaGetLastError();
          return e;
        }
        p.xfrag = ws + L.xfrag;
      } else {
        p.x_raw = x;
        p.x_vec = x_rows_vec(x, m->cols, xl) ? 1u : 0u;
      }
      // the preparation launch, when there is one, precedes the GEMV: launch the GEMV as its
      // programmatic dependent so that its plane copies overlap it
      e = launch_gemv_bulk(p, bp, kd, xl, mixed, prep || (flags & HQB_FLAG_PDL) != 0, st);
      if (e != cudaSuccess) return e;
      return cudaGetLastError();
    }
  }
  const uint8_t* xfrag = static_cast<const uint8_t*>(x);
  const uint32_t xslot16 = xslot_bytes_for(batch, xl);
  // Row-block kernel (uniform prefix, batch <= 8, every warp's activation fragments in its
  // shared memory; it always prepares raw activations itself): the default for small
  // layers, where the stream-K kernel's fixed cost (activation staging, cross-CTA
  // split-row sums) dominates.  Rule, from B200 timings of both kernels: a stream-K CTA
  // would hold u <= kRowsUnitsMax (tile, stage) units, and a row-block warp streams at
  // most u + 2.5 units (its items per CTA times its share of a row block).
  const uint32_t rows_xw = mixed ? 0u : rows_xw_bytes(m->grid_cols, prefix, xslot16);
  const uint64_t all_units = static_cast<uint64_t>(m->grid_rows) * m->grid_cols * prefix;
  const uint64_t warp_units = ((static_cast<uint64_t>(m->grid_rows) * 8 + sms - 1) / sms) *
                              ((static_cast<uint64_t>(m->grid_cols) * prefix + kRowsWarps - 1) / kRowsWarps);
  // With the int8 forms (raw x, batch <= 2) the stream-K kernel also wins once a
  // row-block CTA would take more than two row-block items (B200 timings at 2048..12288
  // rows, prefix 1..4), and at two items once the layer is wider than 32 tile columns
  // (4096x8192: 7.1 / 8.5 against 8.2 / 10.6 us at prefix 1 / 2; 4096x4096 stays with the
  // row-block kernel, 5.9 against 6.1 us at prefix 2).
  const bool i8_form = !mixed && !simt && !x_prepared && batch <= 2 &&
                       !(flags & (HQB_FLAG_RING | HQB_FLAG_F16MMA));
  const uint64_t rows_items_cta = (static_cast<uint64_t>(m->grid_rows) * 8 + sms - 1) / sms;
  const bool rows_small = all_units <= static_cast<uint64_t>(kRowsUnitsMax) * 2 * sms &&
                          warp_units * 2 * sms <= all_units + 5ull * sms &&
                          (!i8_form || rows_items_cta == 1 || (rows_items_cta == 2 && m->grid_cols <= 32));
  // FP32 x at batch <= 2 (int8 limbs) keeps to the lean stream-K kernel unless the row-block
  // kernel is asked for: only limb_item slots keep activations of 2^100 and more exact
  const bool rows_path = !mixed && !simt && batch <= 8 && !(flags & (HQB_FLAG_RING | HQB_FLAG_STREAMK)) &&
                         (x_dtype != HQB_F32 || batch > 2 || x_prepared ||
                          (flags & (HQB_FLAG_ROWBLOCK | HQB_FLAG_F16MMA))) &&
                         (rows_small || (flags & HQB_FLAG_ROWBLOCK)) &&
                         static_cast<uint64_t>(m->grid_rows) * m->grid_cols * kRecordBytes < (1ull << 32) &&
                         kRowsHeadBytes + static_cast<uint64_t>(kRowsWarps) * rows_xw <= kRowsSmemMax;
  // Activation slots a uniform stream-K CTA holds: min(C, its tiles), its tiles at most
  // ceil(units / D) + 1 for units <= ceil(total / G) and any grid G >= min(SMs, total).
  const uint64_t units_cta = (all_units + sms - 1) / sms;
  const uint32_t uniform_res_slots = static_cast<uint32_t>(
      std::min<uint64_t>(m->grid_cols, prefix == 0 ? 1 : (units_cta + prefix - 1) / prefix + 1));
  // int8 activation limbs: raw FP16 or FP32 x, batch <= 2, and the limb slots fit (the row-block
  // kernel's per-warp areas, or the stream-K CTA's resident slots).
  const bool i8_raw = !simt && !x_prepared && batch <= 2 &&
                      !(flags & (HQB_FLAG_RING | HQB_FLAG_F16MMA));
  const bool i8_ok = !mixed && i8_raw;
  // A depth map on the int8 unit kernel (gemv_unit_kernel): its CTAs hold at most
  // ceil(R·C·stage_count / SMs) units, so as many tiles plus one.
  const uint32_t mixed_res_slots = static_cast<uint32_t>(std::min<uint64_t>(
      m->grid_cols, (static_cast<uint64_t>(m->grid_rows) * m->grid_cols * m->stage_count + sms - 1) / sms + 1));
  const bool mx = mixed && i8_raw && static_cast<uint64_t>(mixed_res_slots) * xslot_i8_bytes(batch) <= kXResidentMaxI8;
  const uint32_t rows_xw_i8 = rows_path && i8_ok ? rows_xw_bytes(m->grid_cols, prefix, xslot_i8_bytes(batch)) : 0u;
  const bool rows_i8 = rows_path && i8_ok && kRowsHeadBytes + static_cast<uint64_t>(kRowsWarps) * rows_xw_i8 <= kRowsSmemMax;
  const bool i8 = mx || rows_i8 || (!rows_path && i8_ok &&
                                    static_cast<uint64_t>(uniform_res_slots) * xslot_i8_bytes(batch) <= kXResidentMaxI8);
  const uint32_t res_slots = mx ? mixed_res_slots : uniform_res_slots;
  const uint32_t xslot = i8 ? xslot_i8_bytes(batch) : xslot16;
  const uint64_t x_all_bytes = static_cast<uint64_t>(m->grid_cols) * xslot;
  // stream-K kernels: all fragments resident in shared memory (else the ring kernel)
  const bool streaming = !rows_path && !simt && (i8 || (x_all_bytes <= kXResidentMax && !(flags & HQB_FLAG_RING)));
  // The uniform stream-K kernel builds the fragments of the columns its tiles touch; when
  // CTAs hold more than kFusedTilesMax tiles on average, one preparation launch shared by
  // all is cheaper.
  const uint64_t avg_tiles = static_cast<uint64_t>(m->grid_rows) * m->grid_cols / (static_cast<uint64_t>(sms) * 2);
  const bool fuse_prep = !x_prepared && (rows_path || (streaming && (!mixed || mx) && avg_tiles <= kFusedTilesMax));
  if (!x_prepared && !fuse_prep && info == nullptr) {
    // the int8 stream-K kernels (lean uniform and unit depth-map bodies) read limb_item slots
    e = i8 ? launch_prep_limbs(x, x_dtype, m->cols, batch, ws + L.xfrag, (flags & HQB_FLAG_PDL) != 0, st)
           : launch_prep(x, x_dtype, m->cols, batch, ws + L.xfrag, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return e;
    }
    xfrag = ws + L.xfrag;
  }
  GemvParams p{};
  for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) p.planes[s] = static_cast<const uint8_t*>(m->planes[s]);
  p.depth = depth;
  p.plan = depth_plan;
  p.xfrag = xfrag;
  p.bias = bias;
  p.y = y;
  p.error = reinterpret_cast<int*>(ws);
  p.partials = reinterpret_cast<float*>(ws + L.partials);
  p.counters = reinterpret_cast<uint32_t*>(ws + L.counters);
  p.rows = static_cast<uint32_t>(m->rows);
  p.R = m->grid_rows;
  p.C = m->grid_cols;
  p.prefix = mixed ? 0 : prefix;
  p.stage_count = m->stage_count;
  p.batch = batch;
  p.xslot_bytes = xslot;
  p.bias_dtype = bias_dtype;
  p.y_dtype = y_dtype;
  p.cols = static_cast<uint32_t>(m->cols);
  p.shift_mul = 1u << 24;
  p.pdl = (flags & HQB_FLAG_PDL) ? 1u : 0u;
  if (gather != nullptr) {
    // only the row-block and uniform stream-K kernels gather
    if (!rows_path && !streaming) return HQB_ERR_UNSUPPORTED;
    p.g_world = gather->world;
    p.g_rank = gather->rank;
    p.g_slot_rows = gather->slot_rows;
    for (uint32_t r = 0; r < gather->world; ++r) {
      p.g_peer_y[r] = gather->peer_y[r];
      p.g_peer_flags[r] = gather->peer_flags[r];
    }
    p.g_done = reinterpret_cast<uint32_t*>(ws + L.counters) + m->grid_rows;
  }
  if (fuse_prep) {
    p.x_raw = x;
    p.x_vec = x_rows_vec(x, m->cols, xl) ? 1u : 0u;
  }
  const uint64_t tiles = static_cast<uint64_t>(m->grid_rows) * m->grid_cols;
  p.total = mixed ? 0 : tiles * prefix;
  GemvKernel k = nullptr;
  uint32_t smem = 0, threads = 0;
  uint64_t work = p.total;  // upper bound on useful CTAs
  if (rows_path) {
    p.xw_bytes = rows_i8 ? rows_xw_i8 : rows_xw;
    k = pick_rows_kernel(xl, prefix, batch, rows_i8);
    smem = kRowsHeadBytes + kRowsWarps * p.xw_bytes;
    threads = kRowsThreads;
    work = static_cast<uint64_t>(m->grid_rows) * 8;  // row-block items
  } else {
    k = !streaming ? pick_kernel(batch > 8 ? 2 : 1, xl, simt)
        : mx       ? pick_mixed_i8(batch, xl)
        : mixed    ? pick_stream_kernel(batch > 8 ? 2 : 1, xl)
                   : pick_uniform_kernel(batch > 8 ? 2 : 1, xl, prefix, batch, i8);
    p.x_resident = (i8 || x_all_bytes <= kXResidentMax) ? 1u : 0u;
    p.slot_x_bytes = p.x_resident ? 0u : xslot;
    const RingShape rs = ring_shape(p.slot_x_bytes, mixed ? m->stage_count : prefix,
                                    p.x_resident ? static_cast<uint32_t>(x_all_bytes) : 0u);
    p.ring_slots = rs.slots;
    p.slot_stride = rs.stride;
    p.x_res_slots = res_slots;
    smem = !streaming          ? rs.smem
           : (mixed && !mx)    ? static_cast<uint32_t>(x_all_bytes) + 256
           : i8                ? res_slots * xslot + (kStreamThreads / 32) * 512 + 256  // + limb transpose areas
                               : res_slots * xslot + 256;
    threads = streaming ? kStreamThreads : kGemvThreads;
  }
  const int per_sm = ctas_per_sm(k, smem, device, threads);
  if (per_sm <= 0) return cudaErrorLaunchOutOfResources;
  uint64_t grid = static_cast<uint64_t>(sms) * per_sm;
  if (!mixed) grid = std::max<uint64_t>(1, std::min<uint64_t>(grid, work));
  if (info) {
    const bool self_fin = rows_path || (streaming && (!mixed || mx));
    const bool fix = !self_fin && (mixed || std::min<uint64_t>(grid, p.total) > 1);
    const char* name = rows_path ? "gemv_rows_kernel"
                       : !streaming ? "gemv_kernel"
                       : (mixed && !mx) ? "gemv_stream_kernel"
                       : mx             ? "gemv_unit_kernel"
                                        : "gemv_uniform_kernel";
    return describe(name, (!x_prepared && !fuse_prep ? 1u : 0u) + 1u + (fix ? 1u : 0u), i8, grid, threads, smem);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (flags & HQB_FLAG_PDL) {
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  e = cudaLaunchKernelEx(&cfg, k, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // do not leave a refused launch pending for the next call
    return e;
  }
  // Split tile rows exist whenever more than one CTA shares the work; the row-block and
  // uniform stream-K kernels finish them (or have none) themselves.
  const bool self_finishing = rows_path || (streaming && (!mixed || mx));
  if (!self_finishing && (mixed || std::min<uint64_t>(grid, p.total) > 1)) {
    cudaLaunchConfig_t fc{};
    fc.gridDim = dim3(m->grid_rows);
    fc.blockDim = dim3(256);
    fc.stream = st;
    fc.attrs = attr;
    fc.numAttrs = 1;
    e = cudaLaunchKernelEx(&fc, fixup_kernel, p, static_cast<uint32_t>(grid));
    if (e != cudaSuccess) {
      cudaGetLastError();
      return e;
    }
  }
  return cudaGetLastError();
}

}  // namespace

extern "C" {

HQB_API int hqb_gemv_ex(const hqb_plane_matrix* m, uint32_t prefix, const uint8_t* depth, const uint32_t* depth_plan,
                        const void* x, int x_dtype, uint32_t batch, int x_prepared, const void* bias, int bias_dtype,
                        void* y, int y_dtype, void* workspace, uint64_t workspace_bytes, uint32_t flags,
                        void* stream) {
  return gemv_impl(m, prefix, depth, depth_plan, x, x_dtype, batch, x_prepared, bias, bias_dtype, y, y_dtype,
                   workspace, workspace_bytes, flags, stream, nullptr);
}

HQB_API int hqb_gemv_query(const hqb_plane_matrix* m, uint32_t prefix, int mixed, int x_dtype, uint32_t batch,
                           int x_prepared, uint32_t flags, hqb_launch_info* info) {
  if (info == nullptr) return HQB_ERR_INVALID;
  // stand-in operands: aligned, never dereferenced in a dry run
  static const uint8_t depth_stub[16] = {};
  static const uint32_t plan_stub[4] = {};
  void* const stub = reinterpret_cast<void*>(static_cast<uintptr_t>(4096));
  return gemv_impl(m, prefix, mixed ? depth_stub : nullptr, mixed ? plan_stub : nullptr, stub, x_dtype, batch,
                   x_prepared, nullptr, HQB_F32, stub, HQB_F16, stub, UINT64_MAX, flags, nullptr, nullptr, info);
}

HQB_API int hqb_gemv_gather(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype, uint32_t batch,
                            const void* bias, int bias_dtype, int y_dtype, const hqb_gather* gather,
                            void* workspace, uint64_t workspace_bytes, uint32_t flags, void* stream) {
  if (gather == nullptr) return HQB_ERR_INVALID;
  return gemv_impl(m, prefix, nullptr, nullptr, x, x_dtype, batch, 0, bias, bias_dtype, nullptr, y_dtype, workspace,
                   workspace_bytes, flags, stream, gather);
}

HQB_API int hqb_gather_wait_ex(const uint32_t* flags, uint32_t world, uint32_t* epoch, int* device_flags,
                               uint64_t limit_ns, void* stream) {
  if (flags == nullptr || epoch == nullptr || world == 0 || world > HQB_MAX_PEERS || limit_ns == 0)
    return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  gather_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(flags, world, epoch, device_flags,
                                                      std::min<uint64_t>(limit_ns, kWaitLimitNs));
  return cudaGetLastError();
}

HQB_API int hqb_gather_wait(const uint32_t* flags, uint32_t world, uint32_t* epoch, int* device_flags,
                            void* stream) {
  return hqb_gather_wait_ex(flags, world, epoch, device_flags, kWaitLimitNs, stream);
}

HQB_API int hqb_peer_alloc(uint64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes == 0 || ptr == nullptr || ipc_handle == nullptr) return HQB_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == HQB_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return e;
  }
  *ptr = p;
  return cudaSuccess;
}

HQB_API int hqb_peer_open(const void* ipc_handle, void** ptr) {
  if (ipc_handle == nullptr || ptr == nullptr) return HQB_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

HQB_API int hqb_peer_close(void* ptr) {
  if (ptr == nullptr) return HQB_ERR_INVALID;
  return cudaIpcCloseMemHandle(ptr);
}

HQB_API int hqb_peer_free(void* ptr) {
  if (ptr == nullptr) return HQB_ERR_INVALID;
  return cudaFree(ptr);
}

HQB_API int hqb_gemv_batch(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                           void* stream) {
  if (calls == nullptr || count == 0) return HQB_ERR_INVALID;
  for (uint32_t i = 0; i < count; ++i) {
    const hqb_gemv_call& c = calls[i];
    const int st = gemv_impl(c.m, c.prefix, c.depth, c.depth_plan, c.x, c.x_dtype, c.batch, c.x_prepared, c.bias,
                             c.bias_dtype, c.y, c.y_dtype, workspace, workspace_bytes, c.flags, stream, nullptr);
    if (st != HQB_OK) return st;
  }
  return HQB_OK;
}

}  // extern "C"

namespace {

using GroupKernel = void (*)(GroupParams);

template <int XL, int D>
GroupKernel pick_grouped_d(bool b1) {
  return b1 ? gemv_grouped_kernel<XL, D, true> : gemv_grouped_kernel<XL, D, false>;
}

GroupKernel pick_grouped(uint32_t xl, uint32_t d, bool b1) {
  if (xl == 1) {
    switch (d) {
      case 1: return pick_grouped_d<1, 1>(b1);
      case 2: return pick_grouped_d<1, 2>(b1);
      case 3: return pick_grouped_d<1, 3>(b1);
      default: return pick_grouped_d<1, 4>(b1);
    }
  }
  switch (d) {
    case 1: return pick_grouped_d<2, 1>(b1);
    case 2: return pick_grouped_d<2, 2>(b1);
    case 3: return pick_grouped_d<2, 3>(b1);
    default: return pick_grouped_d<2, 4>(b1);
  }
}

// One grouped launch of independent calls, or HQB_ERR_UNSUPPORTED when they do not share
// the form it needs (uniform prefix, batch <= 2, raw x of one dtype, int8 limbs).
int grouped_launch(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                   void* stream) {
  if (count < 2 || count > kMaxGroup) return HQB_ERR_UNSUPPORTED;
  const hqb_gemv_call& c0 = calls[0];
  const uint32_t d = c0.prefix, batch = c0.batch;
  const int xd = c0.x_dtype;
  const uint32_t bad_flags = HQB_FLAG_SIMT | HQB_FLAG_RING | HQB_FLAG_TCGEN05 | HQB_FLAG_ROWBLOCK | HQB_FLAG_F16MMA |
                             HQB_FLAG_BULK;
  uint32_t maxR = 0, maxC = 0;
  uint64_t units[kMaxGroup], total = 0;
  for (uint32_t i = 0; i < count; ++i) {
    const hqb_gemv_call& c = calls[i];
    if (!plane_matrix_ok(c.m) || c.x == nullptr || c.y == nullptr) return HQB_ERR_INVALID;
    if (c.depth != nullptr || c.depth_plan != nullptr || c.x_prepared || c.prefix != d || d == 0 ||
        d > c.m->stage_count || c.batch != batch || batch == 0 || batch > 2 || c.x_dtype != xd ||
        (c.flags & bad_flags))
      return HQB_ERR_UNSUPPORTED;
    if ((xd != HQB_F16 && xd != HQB_F32) || (c.y_dtype != HQB_F16 && c.y_dtype != HQB_F32)) return HQB_ERR_INVALID;
    if (c.bias != nullptr && c.bias_dtype != HQB_F16 && c.bias_dtype != HQB_F32) return HQB_ERR_INVALID;
    if (!stage_planes_ok(c.m, d)) return HQB_ERR_INVALID;
    maxR = std::max(maxR, c.m->grid_rows);
    maxC = std::max(maxC, c.m->grid_cols);
    units[i] = static_cast<uint64_t>(c.m->grid_rows) * c.m->grid_cols * d;
    total += units[i];
  }
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return HQB_ERR_INVALID;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  const int sms = device_sm_count(device);
  if (sms <= 0) return cudaErrorNoDevice;
  const uint32_t xl = xd == HQB_F32 ? 2 : 1;
  // the grouped launch uses the error word and the partials region (at its offset for the
  // tallest call): the workspace of the call with the most tile rows is large enough
  const WsLayout L = ws_layout(maxR, maxC, batch, xl, sms);
  if (workspace_bytes < L.xfrag) return HQB_ERR_INVALID;
  // CTAs dealt in proportion to each call's units (at least one each)
  const GroupKernel k = pick_grouped(xl, d, batch == 1);
  const uint32_t xslot = xslot_i8_bytes(batch);
  GroupParams gp{};
  gp.count = count;
  uint32_t G = static_cast<uint32_t>(sms) * 2;
  uint32_t res_max = 0;
  for (int attempt = 0; attempt < 2; ++attempt) {
    // CTAs dealt so that every call's CTAs cost about the same: a CTA's time is its units
    // plus the limb columns it builds (each about kLimbColUnits units of streaming time,
    // B200 timelines); bisection on that cost, then the CTAs left over by rounding go to
    // the calls in turn.
    uint32_t gcount[kMaxGroup];
    auto ctas_for = [&](uint32_t i, double cost) -> uint32_t {
      const uint32_t C = calls[i].m->grid_cols;
      uint32_t lo = 1, hi = G;  // smallest g with cost_i(g) <= cost
      while (lo < hi) {
        const uint32_t mid = (lo + hi) / 2;
        const double u = static_cast<double>(units[i]) / mid;
        const double cols = std::min<double>(C, u / d + 1.0);
        if (u + kLimbColUnits * cols <= cost) hi = mid;
        else lo = mid + 1;
      }
      return lo;
    };
    double clo = 0.0, chi = static_cast<double>(total) + kLimbColUnits * maxC + 1.0;
    for (int it = 0; it < 48; ++it) {
      const double mid = 0.5 * (clo + chi);
      uint64_t need = 0;
      for (uint32_t i = 0; i < count; ++i) need += ctas_for(i, mid);
      if (need <= G) chi = mid;
      else clo = mid;
    }
    uint32_t used = 0;
    for (uint32_t i = 0; i < count; ++i) used += (gcount[i] = ctas_for(i, chi));
    for (uint32_t i = 0; used < G; i = (i + 1) % count, ++used) ++gcount[i];
    gp.cta_base[0] = 0;
    for (uint32_t i = 0; i < count; ++i) gp.cta_base[i + 1] = gp.cta_base[i] + gcount[i];
    res_max = 0;
    for (uint32_t i = 0; i < count; ++i) {
      const uint64_t g_i = gp.cta_base[i + 1] - gp.cta_base[i];
      const uint64_t units_cta = (units[i] + g_i - 1) / g_i;
      const uint32_t res = static_cast<uint32_t>(std::min<uint64_t>(calls[i].m->grid_cols, (units_cta + d - 1) / d + 1));
      res_max = std::max(res_max, res);
    }
    if (static_cast<uint64_t>(res_max) * xslot <= kXResidentMaxI8) break;
    if (attempt == 1) return HQB_ERR_UNSUPPORTED;
  }
  const uint32_t smem = res_max * xslot + (kStreamThreads / 32) * 512 + 256;  // + limb transpose areas
  {
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(k), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kXResidentMaxI8 + 4096 + 256));
    int per_sm = 0;
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, static_cast<int>(kStreamThreads), smem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return e;
    }
    if (per_sm < 2) return HQB_ERR_UNSUPPORTED;
  }
  G = gp.cta_base[count];
  if (G > static_cast<uint32_t>(sms) * kMaxCtasPerSm) return HQB_ERR_UNSUPPORTED;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  for (uint32_t i = 0; i < count; ++i) {
    const hqb_gemv_call& c = calls[i];
    GemvParams& p = gp.p[i];
    for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) p.planes[s] = static_cast<const uint8_t*>(c.m->planes[s]);
    p.bias = c.bias;
    p.y = c.y;
    p.error = reinterpret_cast<int*>(ws);
    // each call's CTAs publish split-row words in their own slots of the partials region
    p.partials = reinterpret_cast<float*>(ws + L.partials + static_cast<uint64_t>(gp.cta_base[i]) * batch * 1024);
    p.counters = reinterpret_cast<uint32_t*>(ws + L.counters);
    p.rows = static_cast<uint32_t>(c.m->rows);
    p.R = c.m->grid_rows;
    p.C = c.m->grid_cols;
    p.prefix = d;
    p.stage_count = c.m->stage_count;
    p.batch = batch;
    p.xslot_bytes = xslot;
    p.bias_dtype = c.bias_dtype;
    p.y_dtype = c.y_dtype;
    p.cols = static_cast<uint32_t>(c.m->cols);
    p.shift_mul = 1u << 24;
    p.pdl = (c.flags & HQB_FLAG_PDL) ? 1u : 0u;
    p.x_raw = c.x;
    p.x_vec = x_rows_vec(c.x, c.m->cols, xl) ? 1u : 0u;
    p.total = units[i];
    p.x_res_slots = res_max;
  }
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (calls[0].flags & HQB_FLAG_PDL) {
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  e = cudaLaunchKernelEx(&cfg, k, gp);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  return HQB_OK;
}

}  // namespace

extern "C" {

HQB_API int hqb_gemv_grouped(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                             void* stream) {
  if (calls == nullptr || count == 0) return HQB_ERR_INVALID;
  const int st = grouped_launch(calls, count, workspace, workspace_bytes, stream);
  if (st != HQB_ERR_UNSUPPORTED) return st;
  return hqb_gemv_batch(calls, count, workspace, workspace_bytes, stream);  // one by one
}

HQB_API int hqb_gemv(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype, uint32_t batch,
                     const void* bias, int bias_dtype, void* y, int y_dtype, void* workspace, uint64_t workspace_bytes,
                     void* stream) {
  return hqb_gemv_ex(m, prefix, nullptr, nullptr, x, x_dtype, batch, 0, bias, bias_dtype, y, y_dtype, workspace,
                     workspace_bytes, 0, stream);
}

HQB_API int hqb_gemv_mixed(const hqb_plane_matrix* m, const uint8_t* depth, const uint32_t* depth_plan, const void* x,
                           int x_dtype, uint32_t batch, const void* bias, int bias_dtype, void* y, int y_dtype,
                           void* workspace, uint64_t workspace_bytes, void* stream) {
  if (depth == nullptr || depth_plan == nullptr) return HQB_ERR_INVALID;
  return hqb_gemv_ex(m, 0, depth, depth_plan, x, x_dtype, batch, 0, bias, bias_dtype, y, y_dtype, workspace,
                     workspace_bytes, 0, stream);
}

HQB_API int hqb_decode_planes(const hqb_plane_matrix* m, uint32_t prefix, const uint8_t* depth, float* out,
                              uint64_t out_count, void* stream) {
  if (!plane_matrix_ok(m) || out == nullptr || out_count != m->rows * m->cols) return HQB_ERR_INVALID;
  if (depth == nullptr && prefix > m->stage_count) return HQB_ERR_INVALID;
  if (!stage_planes_ok(m, depth != nullptr ? m->stage_count : prefix)) return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  decode_kernel<<<m->grid_rows * m->grid_cols, 256, 0, as_stream(stream)>>>(*m, prefix, depth, out);
  return cudaGetLastError();
}

}  // extern "C"
