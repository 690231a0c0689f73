// Host-side helpers shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "harpq_b200.h"

namespace hqb {

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

inline bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

inline uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Returns a pending CUDA error without clearing anything else; the caller
// propagates it instead of launching (reference: progressive_gemv.cu:427-433).
inline cudaError_t take_prior_error() { return cudaGetLastError(); }

int device_sm_count(int device);

// The int8-limb GEMV on the reference's raw layout (hqb_raw_i8.cu): 128x128 tiles,
// group 128, prefix 1..4, batch one, FP32 x / y.  HQB_ERR_UNSUPPORTED (nothing
// enqueued) when the geometry, alignment or shared-memory size rules it out.
struct RawI8Launch {
  const hqb_geometry* geometry;
  const uint8_t* codes[HQB_MAX_STAGES];
  const uint16_t* scales[HQB_MAX_STAGES];
  uint32_t prefix;
  const float* x;
  const float* bias;
  float* y;
};
int launch_raw_i8(const RawI8Launch& a, void* stream);
uint32_t raw_i8_smem_bytes(uint64_t padded_cols);

}  // namespace hqb
