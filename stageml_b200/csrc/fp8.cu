// Per-output-channel e4m3 weight quantization (R6, stage 0): one CTA per row,
//   scale[r] = max_c |w[r, c]| / 448   (1 for an all-zero row)
//   q[r, c]  = e4m3(w[r, c] / scale[r]) round-to-nearest-even, saturated to +-448.
// The reference has no FP8 path; its integer per-channel fake quantizer
// (stageml/quant_absint.py:47-82, per_channel with channel_dim=0) is the
// pattern this follows with an e4m3 code book.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ w, int64_t cols,
                                                            uint8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[8];
  const int64_t r = blockIdx.x;
  const T* row = w + r * cols;
  float mx = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += 256) mx = fmaxf(mx, fabsf(to_f32<T>(row[c])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < 8; ++i) m = fmaxf(m, red[i]);
    red[0] = (m > 0.f) ? m / 448.0f : 1.0f;
  }
  __syncthreads();
  const float s = red[0];
  if (threadIdx.x == 0) scale[r] = s;
  for (int64_t c = threadIdx.x; c < cols; c += 256) {
    const float v = to_f32<T>(row[c]) / s;
    q[r * cols + c] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
  }
}

}  // namespace

int launch_quantize_e4m3_rows(const void* w, int dtype, int64_t rows, int64_t cols, uint8_t* q, float* scale,
                              cudaStream_t stream) {
  SB_CHECK_ARG(w && q && scale, "quantize_e4m3_rows: null pointer");
  SB_CHECK_ARG(rows >= 0 && cols >= 0 && rows <= 0x7fffffff, "quantize_e4m3_rows: bad sizes");
  if (rows == 0) return STAGEML_OK;
  if (dtype == STAGEML_F32)
    (quantize_rows_kernel<float><<<(unsigned)rows, 256, 0, stream>>>(static_cast<const float*>(w), cols, q, scale), ::sb::count_launch());
  else if (dtype == STAGEML_BF16)
    (quantize_rows_kernel<bf16><<<(unsigned)rows, 256, 0, stream>>>(static_cast<const bf16*>(w), cols, q, scale), ::sb::count_launch());
  else if (dtype == STAGEML_F16)
    (quantize_rows_kernel<f16><<<(unsigned)rows, 256, 0, stream>>>(static_cast<const f16*>(w), cols, q, scale), ::sb::count_launch());
  else
    return set_error(STAGEML_ERR_INVALID_ARG, "quantize_e4m3_rows: unsupported dtype %d", dtype);
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb
