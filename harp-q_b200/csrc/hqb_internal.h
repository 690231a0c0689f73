// Host-side helpers shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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

}  // namespace hqb
