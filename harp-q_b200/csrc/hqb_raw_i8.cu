// Int8-limb GEMV on the reference's own device layout: the fast kernel behind
// LaunchProgressiveGemv (reference native/src/progressive_gemv.cu:420-439) for
// 128x128 tiles with group 128 (one FP16 scale per row and tile), FP32 x and y.
//
// The reference layout is row-major (progressive_gemv.cu:359-392): row r's codes for the
// 128 columns of tile column c are the 32 bytes at r·padded_cols/4 + 32c, four codes per
// byte (column 4j + m of the byte group at bits 2m, two's complement), and its scale for
// that tile is FP16 element ((r/128)·C + c)·128 + r%128.  Lane (g, q) of a warp that loads
// the 8 bytes at 32c + 8q of rows g and g + 8 holds, word for word, the A fragment of the
// plane layout's m16n8k32 int8-limb step: word 0 covers columns 32q + 4j + m and word 1
// columns 32q + 16 + 4j + m, the columns the limb slot's B fragment of lane q carries
// (limb_item).  An XOR with 0b10 per code turns the two's-complement code into code + 2,
// the plane's stored form.  So the tensor-core step and its exact epilogue are those of
// the plane kernels, applied to the reference's bytes without a repack or a workspace.
//
// Work split (deterministic, no workspace): CTA i of G takes the 16-row blocks i, i + G,
// ...; its 8 warps split the tile columns evenly (warp w: [wC/8, (w+1)C/8)) and stream
// their (block, column) steps through a register ring that runs across blocks.  At each
// block's end the warps' 16 row sums meet in shared memory and are added in warp order,
// then the bias: the bits depend on the shape only, not on the grid.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <type_traits>

#include "harpq_b200.h"
#include "hqb_gemv_common.cuh"
#include "hqb_internal.h"

namespace hqb {
namespace {

constexpr uint32_t kRawWarps = 8;
constexpr uint32_t kRawThreads = kRawWarps * 32;
constexpr uint32_t kRawSlot = kLimbs * 128u + 80u;  // xslot_i8_bytes(1)
constexpr uint32_t kRawWideOff = kLimbs * 128u + 64u;
constexpr uint32_t kRawFixedSmem = 2 * kRawWarps * 16 * 4 + kRawWarps * 512;  // block sums, limb scratch
constexpr uint32_t kRawBar = 1;  // named barrier of the block ends

struct RawI8Params {
  const uint8_t* codes[HQB_MAX_STAGES];
  const uint16_t* scales[HQB_MAX_STAGES];
  const float* x;
  const float* bias;
  float* y;
  uint64_t row_bytes;  // padded_cols / 4
  uint32_t rows, cols;
  uint32_t C;       // tile columns
  uint32_t blocks;  // 16-row blocks, ceil(rows / 16)
  uint32_t x_vec;
};

// Steps kept in flight per warp (D stages each): the register ring of the plane kernels.
template <int D>
struct RawAhead {
  static constexpr int value = D == 1 ? 8 : (D == 2 ? 4 : (D == 3 ? 3 : 2));
};

__device__ __forceinline__ void ld_raw8(uint2& v, const uint8_t* a, uint64_t policy) {
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(v.x), "=r"(v.y)
               : "l"(a), "l"(policy));
}

__device__ __forceinline__ uint32_t ld_raw_scale(const uint16_t* a, uint64_t policy) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;" : "=r"(v) : "l"(a), "l"(policy));
  return v;
}

// Barrier of the block ends.  Warps reach it from different places of the unrolled ring
// (their column counts differ by one), so it is the non-aligned form.
__device__ __forceinline__ void raw_block_bar() {
  asm volatile("barrier.sync %0, %1;" ::"r"(kRawBar), "r"(kRawThreads) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kRawThreads, 2) raw_i8_kernel(const __grid_constant__ RawI8Params p) {
  constexpr int R = RawAhead<D>::value;
  constexpr int CH = TileChains<D>::value;
  constexpr uint32_t kFull = (1u << D) - 1u;
  constexpr uint32_t kFlip = 0xAAAAAAAAu;  // two's-complement code -> code + 2
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const uint32_t C = p.C, G = gridDim.x;
  float* part = reinterpret_cast<float*>(smem + C * kRawSlot);  // [2][warp][16]
  float* scratch = part + 2 * kRawWarps * 16;                   // [warp][128]
  const uint32_t cb = warp * C / kRawWarps, ce = (warp + 1) * C / kRawWarps, nc = ce - cb;
  const uint32_t nblk = blockIdx.x < p.blocks ? (p.blocks - 1 - blockIdx.x) / G + 1 : 0u;
  const uint64_t total = static_cast<uint64_t>(nblk) * nc;  // this warp's steps
  const uint64_t pol = policy_evict_first();
  const uint64_t row8 = 8 * p.row_bytes;

  // Loader position: the step the next refill loads (block ld_blk, tile column ld_c).
  uint32_t ld_blk = blockIdx.x, ld_c = cb, ld_si = 0;
  uint64_t ld_off = 0;
  auto ld_seek = [&]() {
    ld_off = static_cast<uint64_t>(ld_blk * 16 + g) * p.row_bytes + ld_c * 32 + q * 8;
    ld_si = (((ld_blk >> 3) * C + ld_c) << 7) + (ld_blk & 7) * 16 + g;
  };
  ld_seek();
  uint2 clo[R][D], chi[R][D];
  uint32_t slo[R][D], shi[R][D];
  auto refill = [&](int j) {
#pragma unroll
    for (int s = 0; s < D; ++s) {
      const uint8_t* a = p.codes[s] + ld_off;
      ld_raw8(clo[j][s], a, pol);
      ld_raw8(chi[j][s], a + row8, pol);
      const uint16_t* sp = p.scales[s] + ld_si;
      slo[j][s] = ld_raw_scale(sp, pol);
      shi[j][s] = ld_raw_scale(sp + 8, pol);
    }
    if (++ld_c == ce) {
      ld_c = cb;
      ld_blk += G;
      ld_seek();
    } else {
      ld_off += 32;
      ld_si += 128;
    }
  };
#pragma unroll
  for (int j = 0; j < R; ++j)
    if (static_cast<uint64_t>(j) < total) refill(j);

  // Limb slots of every tile column (slot c for column c), built while the first weight
  // loads are in flight.
  {
    GemvParams lp{};
    lp.x_raw = p.x;
    lp.batch = 1;
    lp.cols = p.cols;
    lp.x_vec = p.x_vec;
    lp.C = C;
    lp.xslot_bytes = kRawSlot;
    build_limb_slots<2, kRawWarps>(lp, smem, scratch + warp * 128, ColRanges{0, C - 1, 1, 0}, 0, warp, lane);
  }
  __syncthreads();
  const uint32_t xres_a = smem_u32(smem);
  // Columns whose slot is wide or non-finite (K >= 0 or NaN, limb_item) need the slower
  // epilogue; a warp without any runs its ring without that branch.
  bool any_wide = false;
  for (uint32_t c = cb + lane; c < ce; c += 32)
    any_wide = any_wide || !(__uint_as_float(lds32a(xres_a + c * kRawSlot + kLimbs * 128u + 4u)) < 0.0f);
  any_wide = __any_sync(0xffffffffu, any_wide);

  const XLaneI8 xl8(1u, lane);
  float y[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  uint32_t cur_c = cb, left = nc, blk = blockIdx.x, bi = 0;

  // A block's end: the warp's 16 row sums go to shared memory; after the barrier warp
  // bi % 8 adds the 8 warps' sums in warp order, then the bias, and stores the rows.
  auto block_end = [&]() {
    quad_sum<true>(y);
    float* pp = part + ((bi & 1) * kRawWarps + warp) * 16;
    if (q == 0) {
      pp[g] = y[0][0];
      pp[g + 8] = y[0][2];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) y[0][e] = 0.0f;
    raw_block_bar();
    if (warp == (bi & (kRawWarps - 1)) && lane < 16) {
      const float* pb = part + (bi & 1) * kRawWarps * 16 + lane;
      float s = pb[0];
#pragma unroll
      for (uint32_t w = 1; w < kRawWarps; ++w) s += pb[w * 16];
      const uint32_t row = blk * 16 + lane;
      if (row < p.rows) p.y[row] = p.bias != nullptr ? s + p.bias[row] : s;
    }
    ++bi;
    blk += G;
    cur_c = cb;
    left = nc;
  };

  // One step from ring slot j: tensor-core sums of the D stages, the exact epilogue.
  auto step = [&](int j, auto wide_tag) {
    constexpr bool WIDE = decltype(wide_tag)::value;
    const uint32_t sa = xres_a + cur_c * kRawSlot;
    XFragI8 xf;
    load_limbs<true>(xf, sa + xl8.frag, sa + xl8.cst);
    uint4 wv[D];
    uint32_t sv[D];
#pragma unroll
    for (int s = 0; s < D; ++s) {
      wv[s] = make_uint4(clo[j][s].x ^ kFlip, chi[j][s].x ^ kFlip, clo[j][s].y ^ kFlip, chi[j][s].y ^ kFlip);
      sv[s] = __byte_perm(slo[j][s], shi[j][s], 0x5410);
    }
    uint32_t acc[CH][4];
    bulk_tile_mma<D, false>(wv, xf, acc, kFull);
    if (!WIDE || xf.K[0] < 0.0f) {
      bulk_tile_epilogue<D, true, false>(sv, xf, acc, y, kFull);
    } else {
      const float f0 = __uint_as_float(lds32a(sa + kRawWideOff));
      bulk_tile_epilogue_wide<D, true, false>(sv, xf, acc, y, kFull, f0, 1.0f);
    }
    ++cur_c;
  };

  auto run = [&](auto wide_tag) {
    uint64_t k = 0;
    // steady state: every refill of the group is a step of this warp
    for (; k + 2 * R <= total; k += R) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        step(j, wide_tag);
        refill(j);
        if (--left == 0) block_end();
      }
    }
#pragma unroll
    for (int jj = 0; jj < 2 * R; ++jj) {
      if (k + jj >= total) break;
      step(jj % R, wide_tag);
      if (k + jj + R < total) refill(jj % R);
      if (--left == 0) block_end();
    }
  };
  if (nc == 0) {  // fewer tile columns than warps: this warp only meets the others
    for (uint32_t i = 0; i < nblk; ++i) block_end();
  } else if (any_wide) {
    run(std::true_type{});
  } else {
    run(std::false_type{});
  }
}

using RawKernel = void (*)(RawI8Params);

RawKernel pick_raw(uint32_t prefix) {
  switch (prefix) {
    case 1: return raw_i8_kernel<1>;
    case 2: return raw_i8_kernel<2>;
    case 3: return raw_i8_kernel<3>;
    case 4: return raw_i8_kernel<4>;
    default: return nullptr;
  }
}

// CTAs per SM of a raw kernel at `smem` bytes (0 when it cannot run), cached per device.
int raw_ctas_per_sm(RawKernel k, uint32_t smem, int device) {
  struct Entry {
    RawKernel k;
    uint32_t smem;
    int device, ctas;
  };
  static std::mutex mu;
  static Entry cache[128];
  static int used = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].k == k && cache[i].smem == smem && cache[i].device == device) return cache[i].ctas;
  if (cudaFuncSetAttribute(reinterpret_cast<const void*>(k), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           227 * 1024) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, static_cast<int>(kRawThreads), smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  n = std::min(n, 2);
  if (used < 128) cache[used++] = Entry{k, smem, device, n};
  return n;
}

}  // namespace

uint32_t raw_i8_smem_bytes(uint64_t padded_cols) {
  return static_cast<uint32_t>(padded_cols / 128 * kRawSlot + kRawFixedSmem);
}

int launch_raw_i8(const RawI8Launch& a, void* stream) {
  const hqb_geometry& gm = *a.geometry;
  if (a.prefix < 1 || a.prefix > HQB_MAX_STAGES || gm.tile_rows != 128 || gm.tile_columns != 128 ||
      gm.group_size != 128 || gm.original_rows > 0x7FFFFFF0ull || gm.padded_columns > (1ull << 24))
    return HQB_ERR_UNSUPPORTED;
  const uint64_t C = gm.padded_columns / 128, grid_rows = gm.padded_rows / 128;
  if (grid_rows * C * 128 > 0xFFFFFFFFull) return HQB_ERR_UNSUPPORTED;  // 32-bit scale indices
  for (uint32_t s = 0; s < a.prefix; ++s)
    if ((reinterpret_cast<uintptr_t>(a.codes[s]) & 7u) != 0 || (reinterpret_cast<uintptr_t>(a.scales[s]) & 1u) != 0)
      return HQB_ERR_UNSUPPORTED;
  const uint32_t smem = raw_i8_smem_bytes(gm.padded_columns);
  if (smem > 227u * 1024u) return HQB_ERR_UNSUPPORTED;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) {
    cudaGetLastError();
    return HQB_ERR_UNSUPPORTED;
  }
  const RawKernel k = pick_raw(a.prefix);
  const int per_sm = raw_ctas_per_sm(k, smem, device);
  const int sms = device_sm_count(device);
  if (per_sm < 1 || sms < 1) return HQB_ERR_UNSUPPORTED;
  RawI8Params p{};
  for (uint32_t s = 0; s < a.prefix; ++s) {
    p.codes[s] = a.codes[s];
    p.scales[s] = a.scales[s];
  }
  p.x = a.x;
  p.bias = a.bias;
  p.y = a.y;
  p.row_bytes = gm.padded_columns / 4;
  p.rows = static_cast<uint32_t>(gm.original_rows);
  p.cols = static_cast<uint32_t>(gm.original_columns);
  p.C = static_cast<uint32_t>(C);
  p.blocks = static_cast<uint32_t>((gm.original_rows + 15) / 16);
  p.x_vec = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 && gm.original_columns % 4 == 0;
  const uint32_t grid = std::min<uint32_t>(p.blocks, static_cast<uint32_t>(per_sm * sms));
  k<<<grid, kRawThreads, smem, as_stream(stream)>>>(p);
  return cudaGetLastError();
}

}  // namespace hqb
