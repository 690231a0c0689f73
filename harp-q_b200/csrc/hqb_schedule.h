// Work partition shared by host and device code.
//
// A "unit" is one stage of one 128x128 tile.  Units are ordered (tile_row,
// tile_col, stage) with the stage innermost; a uniform prefix d gives
// grid_rows*grid_cols*d units, a depth map gives Σ depth.  CTA i of G processes the
// contiguous units [start(i), start(i+1)) with start(i) = floor(i*T/G), so every CTA
// streams the same number of bytes (stream-K style).  A tile row split between CTAs
// is finished by whichever contributor arrives last, which sums the contributions in
// CTA order (deterministic).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define HQB_HD __host__ __device__ __forceinline__
#else
#define HQB_HD inline
#endif

namespace hqb {

HQB_HD uint64_t unit_start(uint64_t cta, uint64_t total, uint64_t ctas) {
  return (cta * total) / ctas;
}

// The CTA whose range contains unit u (largest i with start(i) <= u).
HQB_HD uint32_t unit_owner(uint64_t u, uint64_t total, uint64_t ctas) {
  return static_cast<uint32_t>(((u + 1) * ctas - 1) / total);
}

HQB_HD uint32_t clamp_depth(uint32_t d, uint32_t stage_count) {
  return d < 1 ? 1u : (d > stage_count ? stage_count : d);
}

// First unit of tile row r.
HQB_HD uint64_t row_begin(uint32_t r, const uint32_t* plan, uint64_t units_per_row) {
  return plan != nullptr ? static_cast<uint64_t>(plan[r]) : static_cast<uint64_t>(r) * units_per_row;
}

// Tile row containing unit u: uniform division, or binary search in the plan
// (plan[0] = 0, plan[R] = total, non-decreasing).
HQB_HD uint32_t row_of_unit(uint64_t u, const uint32_t* plan, uint32_t rows,
                            uint64_t units_per_row) {
  if (plan == nullptr) return static_cast<uint32_t>(u / units_per_row);
  uint32_t lo = 0, hi = rows;  // invariant: plan[lo] <= u < plan[hi]
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (static_cast<uint64_t>(plan[mid]) <= u) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace hqb
