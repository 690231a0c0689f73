// Prefill (batch >> 16): y[B][rows] = x[B][cols] · W_prefix^T (+ bias) for a resident plane
// matrix, where the batch makes the product a dense contraction worth the tensor cores'
// full rate.  The selected stages are decoded once per call into FP16 weights (row-major
// [rows][cols], in the caller's workspace) and multiplied by cuBLAS with FP16 inputs and
// FP32 accumulation: a plain library GEMM behind the library's own decode.
//
// The decode keeps the reference's per-element arithmetic: code·scale per stage and the
// stage sum in FP32 in stage order (DequantizePrefix, reference native/src/stage_codec.cpp
// :254-272), then one FP16 rounding of that sum.  The prefill GEMM is future work in the
// reference (docs/RESEARCH_PLAN.md:104); this is its first form here.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "harpq_b200.h"
#include "hqb_gemv_common.cuh"
#include "hqb_internal.h"

namespace hqb {
namespace {

// One CTA per tile, one warp per 16-row block (the plane record's own layout): the lane's
// four code words cover rows g and g + 8, columns 32q..32q+15 and 32q+16..32q+31.
__global__ void __launch_bounds__(256) decode_f16_kernel(hqb_plane_matrix m, uint32_t prefix, __half* __restrict__ out) {
  const uint32_t tile = blockIdx.x;
  const uint32_t r = tile / m.grid_cols, c = tile % m.grid_cols;
  const uint32_t rb = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  uint32_t words[HQB_MAX_STAGES][4];
  float sc[HQB_MAX_STAGES][2];
#pragma unroll
  for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) {
    if (s < prefix) {
      const uint8_t* rec = static_cast<const uint8_t*>(m.planes[s]) + static_cast<uint64_t>(tile) * kRecordBytes +
                           rb * kRowBlockBytes;
      const uint4 w = *reinterpret_cast<const uint4*>(rec + lane * 16);
      words[s][0] = w.x;
      words[s][1] = w.y;
      words[s][2] = w.z;
      words[s][3] = w.w;
      const uint32_t pair = *reinterpret_cast<const uint32_t*>(rec + 512 + g * 4);
      sc[s][0] = __half2float(__ushort_as_half(static_cast<unsigned short>(pair & 0xFFFFu)));
      sc[s][1] = __half2float(__ushort_as_half(static_cast<unsigned short>(pair >> 16)));
    }
  }
  const bool vec = (m.cols % 8) == 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t row = static_cast<uint64_t>(r) * 128 + rb * 16 + g + 8 * (i & 1);
    const uint64_t col0 = static_cast<uint64_t>(c) * 128 + 32 * q + 16 * (i >> 1);
    if (row >= m.rows || col0 >= m.cols) continue;
    __half h[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float wsum = 0.0f;
#pragma unroll
      for (uint32_t s = 0; s < HQB_MAX_STAGES; ++s) {
        if (s >= prefix) break;
        // code * scale is exact in FP32 (an FP16 scale times an integer in [-2, 1]), so one
        // fused multiply-add rounds exactly as the separate product and sum do
        const float code = static_cast<float>(static_cast<int>((words[s][i] >> (2 * k)) & 3u) - 2);
        wsum = __fmaf_rn(code, sc[s][i & 1], wsum);
      }
      h[k] = __float2half_rn(wsum);
    }
    __half* dst = out + row * m.cols + col0;
    if (vec && col0 + 16 <= m.cols) {
      reinterpret_cast<uint4*>(dst)[0] = *reinterpret_cast<const uint4*>(&h[0]);
      reinterpret_cast<uint4*>(dst)[1] = *reinterpret_cast<const uint4*>(&h[8]);
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (col0 + k < m.cols) dst[k] = h[k];
    }
  }
}

// y[b][row] (+)= bias[row]; prefix 0 writes bias or zeros.
__global__ void prefill_bias_kernel(void* y, int y_dtype, const void* bias, int bias_dtype, uint32_t rows,
                                    uint32_t batch, int overwrite) {
  const uint64_t n = static_cast<uint64_t>(rows) * batch;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t row = static_cast<uint32_t>(i % rows);
    float b = 0.0f;
    if (bias != nullptr)
      b = bias_dtype == HQB_F32 ? static_cast<const float*>(bias)[row]
                                : __half2float(static_cast<const __half*>(bias)[row]);
    if (y_dtype == HQB_F32) {
      float* yp = static_cast<float*>(y) + i;
      *yp = overwrite ? b : *yp + b;
    } else {
      __half* yp = static_cast<__half*>(y) + i;
      *yp = __float2half_rn(overwrite ? b : __half2float(*yp) + b);
    }
  }
}

// One cuBLAS handle per (host thread, device), created on first use and kept until exit.
cublasHandle_t blas_handle(int device) {
  static thread_local cublasHandle_t handles[64] = {};
  if (device < 0 || device >= 64) return nullptr;
  if (handles[device] == nullptr) {
    cublasHandle_t h = nullptr;
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return nullptr;
    handles[device] = h;
  }
  return handles[device];
}

}  // namespace
}  // namespace hqb

using namespace hqb;

extern "C" {

HQB_API uint64_t hqb_prefill_workspace_bytes(const hqb_plane_matrix* m) {
  if (m == nullptr) return 0;
  return round_up(m->rows * m->cols * 2, 256);
}

HQB_API int hqb_prefill_gemm(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype, uint32_t batch,
                             const void* bias, int bias_dtype, void* y, int y_dtype, void* workspace,
                             uint64_t workspace_bytes, void* stream) {
  if (m == nullptr || x == nullptr || y == nullptr || batch == 0 || m->rows == 0 || m->cols == 0 ||
      m->stage_count == 0 || m->stage_count > HQB_MAX_STAGES || prefix > m->stage_count ||
      m->grid_rows != (m->rows + 127) / 128 || m->grid_cols != (m->cols + 127) / 128)
    return HQB_ERR_INVALID;
  if ((y_dtype != HQB_F16 && y_dtype != HQB_F32) || (bias != nullptr && bias_dtype != HQB_F16 && bias_dtype != HQB_F32))
    return HQB_ERR_INVALID;
  if (x_dtype != HQB_F16) return HQB_ERR_UNSUPPORTED;  // the GEMM takes FP16 activations
  if (m->rows > 0x7FFFFFFFull || m->cols > 0x7FFFFFFFull || batch > 0x7FFFFFFFu) return HQB_ERR_UNSUPPORTED;
  for (uint32_t s = 0; s < prefix; ++s)
    if (m->planes[s] == nullptr || (reinterpret_cast<uintptr_t>(m->planes[s]) & 15u) != 0) return HQB_ERR_INVALID;
  const cudaError_t prior = take_prior_error();
  if (prior != cudaSuccess) return prior;
  cudaStream_t st = as_stream(stream);
  const uint64_t n = m->rows * static_cast<uint64_t>(batch);
  const unsigned fill_blocks = static_cast<unsigned>(n / 256 + 1 < 4096 ? n / 256 + 1 : 4096);
  if (prefix == 0) {
    prefill_bias_kernel<<<fill_blocks, 256, 0, st>>>(y, y_dtype, bias, bias_dtype, static_cast<uint32_t>(m->rows),
                                                     batch, 1);
    return cudaGetLastError();
  }
  if (workspace == nullptr || workspace_bytes < hqb_prefill_workspace_bytes(m) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return HQB_ERR_INVALID;
  __half* w = static_cast<__half*>(workspace);
  decode_f16_kernel<<<m->grid_rows * m->grid_cols, 256, 0, st>>>(*m, prefix, w);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int device = 0;
  e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  cublasHandle_t h = blas_handle(device);
  if (h == nullptr || cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
  const float one = 1.0f, zero = 0.0f;
  const int rows = static_cast<int>(m->rows), cols = static_cast<int>(m->cols), b = static_cast<int>(batch);
  // row-major W[rows][cols] is column-major [cols][rows]: Y_col[rows][B] = W · X_col, the
  // storage of row-major y[B][rows]
  const cublasStatus_t bs =
      cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, rows, b, cols, &one, w, CUDA_R_16F, cols, x, CUDA_R_16F, cols, &zero, y,
                   y_dtype == HQB_F32 ? CUDA_R_32F : CUDA_R_16F, rows, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (bs != CUBLAS_STATUS_SUCCESS) return cudaErrorUnknown;
  if (bias != nullptr) {
    prefill_bias_kernel<<<fill_blocks, 256, 0, st>>>(y, y_dtype, bias, bias_dtype, static_cast<uint32_t>(m->rows),
                                                     batch, 0);
    return cudaGetLastError();
  }
  return cudaSuccess;
}

}  // extern "C"
