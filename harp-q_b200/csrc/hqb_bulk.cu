// Bulk-copy pipelined plane GEMV on int8 activation limbs (batch <= 2), sm_100a.
//
//   gemv_bulk_kernel<D, B1, XL, MX>
//     D   selected prefix depth (MX: 4, each tile cut to its own depth)
//     B1  batch one (only accumulator column 0 of each limb pair is stored)
//     XL  1: FP16 activations, 2: FP32 activations (the limbs are built from either)
//     MX  per-tile depth map
//
// Work partition: the stream-K split of the (tile, stage) units over the CTAs, tiles
// walked in descending order, split tile rows published and summed through the
// workspace -- the same partition, arithmetic and output order as the register-ring
// stream-K kernel in hqb_plane.cu.  What differs is how plane bytes reach the tensor
// cores:
//
//   * warp kBulkConsumers (the producer; one lane issues) streams the CTA's tiles into a
//     shared-memory ring of `slots` chunks with 1-D bulk copies (cp.async.bulk, global ->
//     shared, completion on an mbarrier, L2 evict-first; never multicast).  A chunk holds
//     `chunk_tiles` consecutive walk tiles of every selected stage, laid out
//     [stage][tile][4352 B], so each stage of a chunk is ONE contiguous copy of up to
//     ~20-48 KB out of that stage's plane.  B200 timings of this copy pattern: copies
//     of >= 16 KB with 2-3 chunks of 32-48 KB in flight per CTA stream at 5-7 TB/s,
//     while copies of a few KB stall on a per-copy cost; so chunks are large and there
//     are few of them.
//   * the copies are issued before griddepcontrol.wait: under programmatic dependent
//     launch a GEMV fills its ring while the previous kernel of the stream finishes.
//   * warps 0..7 (the consumers) wait for a chunk, then warp w multiplies row block w
//     (tile rows 16w..16w+15) of each of its tiles: one 16-byte shared-memory load of
//     codes and one 4-byte load of the scale pair per lane and stage, the int8-limb
//     m16n8k32 MMAs and the two-FMA epilogue of the stream-K kernel, then frees the
//     chunk (one mbarrier arrival per warp).
//   * per-tile stage masks (the CTA's range ends; with a depth map the tile's depth)
//     come from the producer through a 16-byte word per chunk slot; a stage a tile does
//     not select is not copied, and its scale reads as 0.
//
// Activation limbs: built by the consumer warps from raw x after griddepcontrol.wait
// (x_raw), or copied from a prepared limb buffer by the producer (one or two bulk
// copies, also after the wait) for layers whose CTAs touch many tile columns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "harpq_b200.h"
#include "hqb_device.cuh"
#include "hqb_gemv_common.cuh"
#include "hqb_internal.h"
#include "hqb_schedule.h"

namespace hqb {

constexpr uint32_t kBulkConsumers = 8;  // consumer warp w owns row block w of every tile
constexpr uint32_t kBulkThreads = (kBulkConsumers + 1) * 32;
constexpr uint32_t kBulkMaxSlots = 8;
constexpr uint32_t kBulkMaxChunkTiles = 16;  // one 16-byte mask word per slot
// shared-memory head: full[8], empty[8], xbar, masks[8][16 B]
constexpr uint32_t kBulkHeadBytes = 512;
constexpr uint32_t kBulkConsumerBar = 1;  // named barrier of the consumer warps

// Walk tiles per ring chunk for each slot depth (stage slots per tile): chunks of about
// 40-52 KB, each stage of a chunk one contiguous copy.
template <int SD>
struct BulkTiles {
  static constexpr uint32_t value = SD == 1 ? 10 : (SD == 2 ? 5 : 3);
};
static_assert(BulkTiles<1>::value <= kBulkMaxChunkTiles && BulkTiles<2>::value <= kBulkMaxChunkTiles,
              "one 16-byte mask word per chunk");
__host__ __device__ constexpr uint32_t bulk_tiles(uint32_t slot_depth) {
  return slot_depth == 1 ? 10u : (slot_depth == 2 ? 5u : 3u);
}

// Word of a chunk's 16-byte mask vector holding tile slot i's byte (selects, no local array).
__device__ __forceinline__ uint32_t bulk_mask_word(const uint4& mw, uint32_t i) {
  return i < 8 ? (i < 4 ? mw.x : mw.y) : (i < 12 ? mw.z : mw.w);
}

// x [batch][cols] -> one limb slot per 128-column tile (limb_item), one warp per (tile
// column, batch row) item: the prepared limbs of the bulk kernel's copied-limb mode.
template <typename XT>
__global__ void __launch_bounds__(128) prep_limbs_kernel(const XT* __restrict__ x, uint32_t cols, uint32_t batch,
                                                         uint32_t C, uint8_t* __restrict__ xfrag, uint32_t xslot) {
  griddep_launch_dependents();
  griddep_wait();  // x may come from the preceding kernel
  const uint32_t item = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= C * batch) return;  // the whole warp leaves together
  const uint32_t c = item / batch, b = item - c * batch;
  float v[4];
  limb_load<XT>(x + static_cast<uint64_t>(b) * cols, c, cols, lane, v);
  limb_item(v, xfrag + static_cast<uint64_t>(c) * xslot, b, batch, lane);
}

// Fused all-gather completion for the consumer warps only (the producer warp has left).
__device__ __forceinline__ void bulk_gather_signal(const GemvParams& p, uint32_t ctas) {
  named_bar_sync(kBulkConsumerBar, kBulkConsumers * 32);
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atom_add_acq_rel_gpu(p.g_done, 1u) == ctas - 1) {
      *p.g_done = 0u;
      for (uint32_t r = 0; r < p.g_world; ++r) red_add_release_sys(p.g_peer_flags[r] + p.g_rank, 1u);
    }
  }
}

template <int D, bool B1, int XL, bool MX>
__global__ void __launch_bounds__(kBulkThreads, 2) gemv_bulk_kernel(const __grid_constant__ GemvParams p) {
  static_assert(!MX || D == HQB_MAX_STAGES, "depth maps run at depth 4");
  constexpr uint32_t kFull = (1u << D) - 1u;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kBulkMaxSlots;
  uint64_t* xbar = empty + kBulkMaxSlots;
  uint8_t* masks = smem + 256;  // [slot][16]
  uint8_t* ring = smem + kBulkHeadBytes;
  const uint32_t S = p.ring_slots, N = p.chunk_tiles, chunk_bytes = p.slot_stride;
  uint8_t* xres = ring + S * chunk_bytes;
  const uint32_t cta = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;

  MixedRange rg{};
  if constexpr (MX) {
    rg = mixed_range(p, cta, lane);
  } else {
    rg.total = p.total;
    rg.ctas = static_cast<uint32_t>(rg.total < gridDim.x ? rg.total : gridDim.x);
    if (cta < rg.ctas) {
      if (rg.total * (rg.ctas + 1) <= 0xffffffffull) {  // 32-bit divisions (the usual case)
        const uint32_t T = static_cast<uint32_t>(rg.total);
        rg.u0 = (cta * T) / rg.ctas;
        rg.u1 = ((cta + 1) * T) / rg.ctas;
      } else {
        rg.u0 = unit_start(cta, rg.total, rg.ctas);
        rg.u1 = unit_start(cta + 1, rg.total, rg.ctas);
      }
      const uint32_t a = static_cast<uint32_t>(rg.u0), z = static_cast<uint32_t>(rg.u1 - 1);
      rg.t0 = a / D;
      rg.s0 = a - rg.t0 * D;
      rg.t_end = z / D;
      rg.s_end = z - rg.t_end * D + 1;
      rg.rb_first = static_cast<uint64_t>(rg.t0 / p.C) * p.C * D;
      rg.re_last = static_cast<uint64_t>(rg.t_end / p.C + 1) * p.C * D;
    }
  }
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kBulkMaxSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kBulkConsumers);
    }
    mbar_init(xbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  griddep_launch_dependents();  // a following PDL kernel may start filling its own ring
  const uint32_t ctas = rg.ctas;
  if (cta >= ctas) return;
  const uint32_t t0 = rg.t0, t_end = rg.t_end;
  const uint32_t ntiles = t_end - t0 + 1;
  const uint32_t nchunks = (ntiles + N - 1) / N;
  const uint32_t mask_first = kFull & ~((1u << rg.s0) - 1u), mask_last = (1u << rg.s_end) - 1u;
  const bool x_copy = p.x_raw == nullptr;  // limbs come from a prepared buffer
  const uint32_t c_first = t0 % p.C;
  const ColRanges cr = needed_columns(t0, t_end, p.C);

  if (warp == kBulkConsumers) {
    // ---------------- producer warp ----------------
    const uint64_t l2_first = policy_evict_first();
    // Prepared limbs (x_copy) may be written by the preceding kernel: they are copied
    // after griddepcontrol.wait, once the first `S` chunks of planes are on their way.
    auto issue_x = [&]() {
      griddep_wait();
      if (lane != 0) return;
      const uint32_t xs = p.xslot_bytes;
      const uint64_t keep = policy_evict_last();
      // columns [a, b] land at resident slots (c - c_first) mod C: contiguous on either
      // side of c_first
      auto copy_cols = [&](uint32_t a, uint32_t b) {
        if (a < c_first && b >= c_first) {
          bulk_load(xres + (a + p.C - c_first) * xs, p.xfrag + static_cast<uint64_t>(a) * xs, (c_first - a) * xs,
                    xbar, keep);
          a = c_first;
        }
        bulk_load(xres + resident_slot(a, c_first, p.C) * xs, p.xfrag + static_cast<uint64_t>(a) * xs,
                  (b - a + 1) * xs, xbar, keep);
      };
      const uint32_t na = cr.a1 - cr.a0 + 1, nb = cr.b1 >= cr.b0 ? cr.b1 - cr.b0 + 1 : 0;
      mbar_expect_tx(xbar, (na + nb) * xs);
      copy_cols(cr.a0, cr.a1);
      if (nb) copy_cols(cr.b0, cr.b1);
    };
    uint32_t issued = 0;
    for (uint32_t k = 0; k < nchunks; ++k) {
      const uint32_t slot = k % S;
      if (k == S && x_copy) issue_x();
      bool ok = true;
      if (lane == 0 && k >= S) ok = mbar_wait(&empty[slot], ((k / S) - 1) & 1, p.error);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      // stage masks of the chunk's walk tiles j (tile t_end - (kk0 + j), smem index N-1-j)
      const uint32_t kk0 = k * N, nhere = min(N, ntiles - kk0);
      uint32_t m = 0;
      if (lane < nhere) {
        const uint32_t kk = kk0 + lane;
        m = kFull;
        if constexpr (MX) m = (1u << clamp_depth(__ldg(p.depth + (t_end - kk)), p.stage_count)) - 1u;
        if (kk == 0) m &= mask_last;
        if (kk == ntiles - 1) m &= mask_first;
        masks[slot * 16 + (N - 1 - lane)] = static_cast<uint8_t>(m);
      }
      uint32_t bits[D];
      uint32_t bytes = 0;
#pragma unroll
      for (int s = 0; s < D; ++s) {
        bits[s] = __ballot_sync(0xffffffffu, (m >> s) & 1u);
        bytes += __popc(bits[s]) * kRecordBytes;
      }
      __syncwarp();  // mask bytes written before the arrival that publishes them
      if (lane == 0) {
        mbar_expect_tx(&full[slot], bytes);
        uint8_t* dst = ring + slot * chunk_bytes;
        // smem index of tile t in this chunk: t - (t_end + 1 - (kk0 + N)) = N-1-j
#pragma unroll
        for (int s = 0; s < D; ++s) {
          uint32_t b = bits[s];
          while (b != 0) {  // runs of consecutive walk tiles j .. j+run-1 (descending tiles)
            const uint32_t j = __ffs(b) - 1;
            const uint32_t run = __ffs(~(b >> j)) - 1;  // N <= 16: bits past the chunk are clear
            b &= ~(((1u << run) - 1u) << j);
            const uint32_t t_lo = t_end - (kk0 + j + run - 1);  // lowest tile of the run
            const uint32_t i = N - 1 - (j + run - 1);           // its smem index
            bulk_load(dst + (s * N + i) * kRecordBytes, p.planes[s] + static_cast<uint64_t>(t_lo) * kRecordBytes,
                      run * kRecordBytes, &full[slot], l2_first);
          }
        }
      }
      issued = k + 1;
    }
    if (x_copy && nchunks <= S) issue_x();
    // every copy issued must land before this CTA may exit
    if (lane == 0) {
      for (uint32_t j = issued > S ? issued - S : 0; j < issued; ++j) mbar_wait(&full[j % S], (j / S) & 1, p.error);
      if (x_copy) mbar_wait(xbar, 0, p.error);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  griddep_wait();  // x, y, the workspace: written or read by the preceding kernel
  // A wait that runs out (HQB_DEVERR_TIMEOUT) ends this warp's work but not the warp:
  // every consumer warp still reaches the barriers below.
  bool alive = true;
  const bool x_ok = min(p.C, ntiles) <= p.x_res_slots;
  if (!x_ok && threadIdx.x == 0) atomicOr(p.error, HQB_DEVERR_LAUNCH);  // smem sized for fewer slots
  if (x_copy) {
    alive = mbar_wait(xbar, 0, p.error);
  } else if (x_ok) {
    build_limb_slots<XL, kBulkConsumers>(p, xres,
                                         reinterpret_cast<float*>(xres + p.x_res_slots * p.xslot_bytes) + warp * 128,
                                         cr, c_first, warp, lane);
    named_bar_sync(kBulkConsumerBar, kBulkConsumers * 32);
  }
  constexpr uint32_t NT = BulkTiles<MX ? HQB_MAX_STAGES : D>::value;
  constexpr uint32_t XS = kLimbs * (B1 ? 1u : 2u) * 128u + 80u;  // xslot_i8_bytes(batch)
  constexpr uint32_t kWideOff = kLimbs * (B1 ? 1u : 2u) * 128u + 64u;
  constexpr int CH = TileChains<D>::value;
  const uint32_t C = p.C;
  const XLaneI8 xl8(B1 ? 1u : 2u, lane);
  const uint32_t xres_a = smem_u32(xres);
  const uint32_t ring_a = smem_u32(ring) + warp * kRowBlockBytes + lane * 16;
  const uint32_t scale_rel = 512 + g * 4 - lane * 16;  // scale pair relative to the lane's codes
  uint32_t xidx = resident_slot(t_end % C, c_first, C);  // resident limb slot of the current tile
  uint32_t row = t_end / C;
  uint32_t left = t_end % C + 1;  // tiles of the current row still ahead (may run past ntiles)
  float y[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  float kept[1][4];
  bool keep = false;
  const uint32_t row_first = t0 / C, row_last = t_end / C;
  const uint64_t u0 = rg.u0, u1 = rg.u1;
  const uint32_t rit0 = warp * 16 + g;

  // Math of one tile (records w/sc in registers, limb slot at shared address xa).
  auto tile_math = [&](const uint4 (&w)[D], const uint32_t (&sc)[D], uint32_t live, uint32_t xa) {
    XFragI8 xf;
    load_limbs<B1>(xf, xa + xl8.frag, xa + xl8.cst);
    uint32_t acc[CH][4];
    bulk_tile_mma<D, MX>(w, xf, acc, live);
    if (xf.K[0] < 0.0f && (B1 || xf.K[1] < 0.0f)) {
      bulk_tile_epilogue<D, B1, MX>(sc, xf, acc, y, live);
    } else {
      const float f0 = __uint_as_float(lds32a(xa + kWideOff)), f1 = B1 ? 1.0f : __uint_as_float(lds32a(xa + kWideOff + 4));
      bulk_tile_epilogue_wide<D, B1, MX>(sc, xf, acc, y, live, f0, f1);
    }
  };
  // After walk tile kk: at the end of a tile row (its column 0) or of the CTA's range the
  // row's sums are stored, published for a later CTA, or kept to be finished last.
  auto row_end = [&](uint32_t kk) {
    if (--left == 0 || kk + 1 == ntiles) {
      quad_sum<B1>(y);
      const uint64_t rb = row == row_first ? rg.rb_first : u0, re = row == row_last ? rg.re_last : u1;
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
    }
  };

  for (uint32_t k = 0; alive && x_ok && k < nchunks; ++k) {
    const uint32_t slot = k % S;
    if (!mbar_wait(&full[slot], (k / S) & 1, p.error)) {
      alive = false;
      break;
    }
    const uint32_t base = ring_a + slot * chunk_bytes;
    const uint32_t kk0 = k * NT, nhere = min(NT, ntiles - kk0);
    if (!MX && nhere == NT && kk0 != 0 && kk0 + NT < ntiles && left > NT && xidx + 1 >= NT) {
      // A whole chunk of full-depth tiles inside one tile row, neither end of the CTA's
      // range, no wrap of the limb slots: every record into registers first, then the math
      // of all its tiles with no branch between them, so the shared-memory loads of later
      // tiles overlap the MMA chains of earlier ones.
      uint4 w[NT][D];
      uint32_t sc[NT][D];
#pragma unroll
      for (uint32_t j = 0; j < NT; ++j)
#pragma unroll
        for (int s = 0; s < D; ++s) {
          const uint32_t a = base + (s * NT + (NT - 1 - j)) * kRecordBytes;
          w[j][s] = lds128a(a);
          sc[j][s] = lds32a(a + scale_rel);
        }
      const uint32_t xa0 = xres_a + xidx * XS;
#pragma unroll
      for (uint32_t j = 0; j < NT; ++j) tile_math(w[j], sc[j], (1u << D) - 1u, xa0 - j * XS);
      left -= NT;
      xidx = xidx >= NT ? xidx - NT : xidx + C - NT;
    } else {
      // Chunks at a row end or at an end of the CTA's range, and depth maps: tile by tile,
      // stages the tile does not select read as scale 0 (with a depth map: skipped).
      const uint4 mw = lds128(masks + slot * 16);
      for (uint32_t j = 0; j < nhere; ++j) {
        const uint32_t i = NT - 1 - j;
        const uint32_t live = (bulk_mask_word(mw, i) >> (8 * (i & 3))) & 0xffu;
        uint4 w[D];
        uint32_t sc[D];
#pragma unroll
        for (int s = 0; s < D; ++s) {
          const uint32_t a = base + (s * NT + i) * kRecordBytes;
          if (MX && !((live >> s) & 1u)) {
            w[s] = make_uint4(0u, 0u, 0u, 0u);
            sc[s] = 0u;
          } else {
            w[s] = lds128a(a);
            sc[s] = ((live >> s) & 1u) ? lds32a(a + scale_rel) : 0u;
          }
        }
        tile_math(w, sc, live, xres_a + xidx * XS);
        row_end(kk0 + j);
        xidx = xidx == 0 ? C - 1 : xidx - 1;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  if (!x_ok) {  // drain the ring so that the producer's waits end
    for (uint32_t k = 0; alive && k < nchunks; ++k) {
      const uint32_t slot = k % S;
      alive = mbar_wait(&full[slot], (k / S) & 1, p.error);
      __syncwarp();
      if (alive && lane == 0) mbar_arrive(&empty[slot]);
    }
  }
  if (keep && alive) reduce_split_row<1, B1>(p, row_first, rg.rb_first, rg.total, ctas, cta, kept, rit0, q);
  if (p.g_world > 1) bulk_gather_signal(p, ctas);
}

// ---------------------------------------------------------------------------------------
// host side

namespace {

template <bool B1, int XL, bool MX>
GemvKernel bulk_kernel_for(uint32_t d) {
  if constexpr (MX) {
    return gemv_bulk_kernel<HQB_MAX_STAGES, B1, XL, true>;
  } else {
    switch (d) {
      case 1: return gemv_bulk_kernel<1, B1, XL, false>;
      case 2: return gemv_bulk_kernel<2, B1, XL, false>;
      case 3: return gemv_bulk_kernel<3, B1, XL, false>;
      default: return gemv_bulk_kernel<4, B1, XL, false>;
    }
  }
}

GemvKernel pick_bulk(uint32_t d, uint32_t batch, uint32_t xl, bool mx) {
  if (mx) {
    if (xl == 1) return batch == 1 ? bulk_kernel_for<true, 1, true>(d) : bulk_kernel_for<false, 1, true>(d);
    return batch == 1 ? bulk_kernel_for<true, 2, true>(d) : bulk_kernel_for<false, 2, true>(d);
  }
  if (xl == 1) return batch == 1 ? bulk_kernel_for<true, 1, false>(d) : bulk_kernel_for<false, 1, false>(d);
  return batch == 1 ? bulk_kernel_for<true, 2, false>(d) : bulk_kernel_for<false, 2, false>(d);
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v != nullptr && *v != '\0' ? std::atoi(v) : dflt;
}

}  // namespace

// Shape of one bulk launch: CTAs per SM, ring slots, tiles per chunk, shared memory.
// tiles: R*C; depth: the uniform prefix, or the stage count for a depth map (mixed),
// whose unit total is known only on the device and is bounded by tiles*depth.
BulkPlan bulk_plan(uint64_t tiles, uint32_t depth, bool mixed, uint32_t C, uint32_t xslot, int sms) {
  BulkPlan b{};
  const uint64_t units = tiles * depth;
  static const int force_ctas = env_int("HQB_BULK_CTAS_PER_SM", 0);
  static const int force_slots = env_int("HQB_BULK_SLOTS", 0);
  // chunk slots per tile: the selected stages, or all four with a depth map
  const uint32_t slot_stages = mixed ? HQB_MAX_STAGES : depth;
  const uint32_t n = bulk_tiles(slot_stages);  // the kernel's compile-time chunk
  // Two CTAs per SM (two producers, 16 consumer warps) wherever their shared memory fits;
  // one CTA with a deeper ring otherwise (B200 timings).
  uint32_t per_sm = 2;
  if (force_ctas == 1 || force_ctas == 2) per_sm = static_cast<uint32_t>(force_ctas);
  for (;;) {
    uint32_t slots = per_sm == 2 ? 2u : 3u;
    if (force_slots >= 2 && force_slots <= static_cast<int>(kBulkMaxSlots)) slots = static_cast<uint32_t>(force_slots);
    const uint32_t grid = static_cast<uint32_t>(
        mixed ? static_cast<uint64_t>(sms) * per_sm
              : std::max<uint64_t>(1, std::min<uint64_t>(units, static_cast<uint64_t>(sms) * per_sm)));
    // tiles a CTA range can touch: ceil(units / G) + 1 for a uniform prefix (each tile holds
    // `depth` units); with a depth map a unit may be a whole tile
    const uint64_t units_cta = (units + grid - 1) / grid;
    const uint64_t tiles_cta = mixed ? units_cta + 1 : (units_cta + depth - 1) / depth + 1;
    const uint32_t res_slots = static_cast<uint32_t>(std::min<uint64_t>(C, tiles_cta));
    const uint64_t chunks_cta = (tiles_cta + n - 1) / n;
    if (slots > chunks_cta) slots = static_cast<uint32_t>(std::max<uint64_t>(2, chunks_cta));
    b.grid = grid;
    b.per_sm = per_sm;
    b.slots = slots;
    b.chunk_tiles = n;
    b.chunk_bytes = n * slot_stages * kRecordBytes;
    b.res_slots = res_slots;
    // + the consumer warps' limb transpose areas (512 B each)
    b.smem = kBulkHeadBytes + slots * b.chunk_bytes + res_slots * xslot + kBulkConsumers * 512u;
    // two CTAs share an SM's 228 KB (1 KB of it reserved per CTA)
    if (per_sm == 2 && b.smem > 113u * 1024u && force_ctas != 2) {
      per_sm = 1;
      continue;
    }
    return b;
  }
}

uint32_t bulk_smem_max() { return 227u * 1024u; }

cudaError_t launch_prep_limbs(const void* x, int x_dtype, uint64_t cols, uint32_t batch, void* xfrag, bool pdl,
                              cudaStream_t st) {
  const uint32_t C = static_cast<uint32_t>((cols + 127) / 128);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((C * batch + 3) / 4);  // one warp per (tile column, batch row)
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (pdl) {
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e;
  if (x_dtype == HQB_F32)
    e = cudaLaunchKernelEx(&cfg, prep_limbs_kernel<float>, static_cast<const float*>(x), static_cast<uint32_t>(cols),
                           batch, C, static_cast<uint8_t*>(xfrag), xslot_i8_bytes(batch));
  else
    e = cudaLaunchKernelEx(&cfg, prep_limbs_kernel<__half>, static_cast<const __half*>(x),
                           static_cast<uint32_t>(cols), batch, C, static_cast<uint8_t*>(xfrag), xslot_i8_bytes(batch));
  if (e != cudaSuccess) cudaGetLastError();
  return e;
}

cudaError_t launch_gemv_bulk(GemvParams p, const BulkPlan& b, uint32_t depth, uint32_t xl, bool mx, bool pdl,
                             cudaStream_t st) {
  if (p.x_raw == nullptr) xl = 1;  // prepared limbs: one slot format for FP16 and FP32 x
  GemvKernel k = pick_bulk(depth, p.batch, xl, mx);
  {
    static std::mutex mu;
    static GemvKernel done[64];
    static int used = 0;
    std::lock_guard<std::mutex> lock(mu);
    bool have = false;
    for (int i = 0; i < used; ++i) have = have || done[i] == k;
    if (!have) {
      const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(k),
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(bulk_smem_max()));
      if (e != cudaSuccess) {
        cudaGetLastError();
        return e;
      }
      if (used < 64) done[used++] = k;
    }
  }
  p.ring_slots = b.slots;
  p.chunk_tiles = b.chunk_tiles;
  p.slot_stride = b.chunk_bytes;
  p.x_res_slots = b.res_slots;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(b.grid);
  cfg.blockDim = dim3(kBulkThreads);
  cfg.dynamicSmemBytes = b.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (pdl) {
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  return cudaSuccess;
}

}  // namespace hqb
