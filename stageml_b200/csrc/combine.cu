// Combine (R2, second half): out[t, :] = sum_j Y[pair_row[t*kk + j], :], the
// routing weight already applied by the down-projection epilogue. This is the
// out.index_add_(0, index, y * gates) of RequestExecutor.dynamic_one
// (benchmarks/multitenant_bta_system_bench.py:413) done once per token with a
// fixed slot order (fp32 sum, one rounding), so it is deterministic.
#include "common.cuh"
#include "host_util.h"
#include "kernels.h"

namespace sb {
namespace {

template <typename T>
__global__ void combine_kernel(const T* __restrict__ y, const int32_t* __restrict__ pair_row, int T_, int kk, int H,
                               T* __restrict__ out, const int32_t* __restrict__ T_dev, int t_base) {
  pdl_wait();  // y comes from the previous kernel
  const int t = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (t >= T_ || c >= H) return;
  if (T_dev && t_base + t >= *T_dev) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int j = 0; j < kk; ++j) {
    const int row = pair_row[(int64_t)t * kk + j];
    if (row < 0) continue;
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(y + (int64_t)row * H + c));
    float f[8];
    unpack8<T>(u, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += f[i];
  }
  *reinterpret_cast<uint4*>(out + (int64_t)t * H + c) = pack8<T>(acc);
}

__global__ void validate_tenants_kernel(const int32_t* __restrict__ in, int64_t n, int n_tenants,
                                        int32_t* __restrict__ out, int32_t* status) {
  pdl_wait();  // the ids may come from the previous kernel
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int v = in ? in[i] : -1;
  if (v < -1 || v >= n_tenants) {
    if (status) atomicCAS(status, 0, (int)kDevBadIndex);
    v = -1;
  }
  out[i] = v;
}

// Rows of a one-expert top-1 layer taken in token order (no permutation): the
// validated tenant of each row and the factor the down projection applies, the
// routing weight, or 0 for a token whose expert id or tenant is out of range (the
// permuted path drops that pair, leaving a zero output row).
__global__ void direct_rows_kernel(const void* __restrict__ ids, int ids_i64, const void* __restrict__ weights,
                                   int weights_dtype, const int32_t* __restrict__ tenant_ids, int n_tenants, int64_t T,
                                   int32_t* __restrict__ row_tenant, float* __restrict__ row_scale, int32_t* status) {
  pdl_wait();  // the ids may come from the previous kernel
  pdl_trigger();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  bool bad = false;
  if (ids) {
    const int64_t e = ids_i64 ? static_cast<const int64_t*>(ids)[t] : (int64_t) static_cast<const int32_t*>(ids)[t];
    bad = e != 0;
  }
  int tn = tenant_ids ? tenant_ids[t] : -1;
  if (tn < -1 || tn >= n_tenants) {
    bad = true;
    tn = -1;
  }
  float w = 1.f;
  if (weights) {
    if (weights_dtype == STAGEML_BF16)
      w = __bfloat162float(static_cast<const bf16*>(weights)[t]);
    else if (weights_dtype == STAGEML_F16)
      w = __half2float(static_cast<const f16*>(weights)[t]);
    else
      w = static_cast<const float*>(weights)[t];
  }
  if (bad && status) atomicCAS(status, 0, (int)kDevBadIndex);
  row_tenant[t] = bad ? -1 : tn;
  row_scale[t] = bad ? 0.f : w;
}

}  // namespace

int launch_direct_rows(const void* ids, int ids_dtype, const void* weights, int weights_dtype, const int32_t* tenant_ids,
                       int n_tenants, int64_t T, int32_t* row_tenant, float* row_scale, int32_t* status,
                       cudaStream_t stream, bool pdl) {
  if (T == 0) return STAGEML_OK;
  SB_CUDA_CHECK(launch_kernel(direct_rows_kernel, dim3((unsigned)((T + 255) / 256)), dim3(256), 0, stream, pdl, ids,
                              ids_dtype == STAGEML_I64 ? 1 : 0, weights, weights_dtype, tenant_ids, n_tenants, T,
                              row_tenant, row_scale, status));
  ::sb::count_launch();
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

int launch_combine(const void* y, const int32_t* pair_row, int T_, int kk, int H, int dtype_bf16, void* out,
                   cudaStream_t stream, const int32_t* T_dev, bool pdl) {
  SB_CHECK_ARG(H % 8 == 0, "combine: H=%d must be a multiple of 8", H);
  if (T_ == 0 || H == 0) return STAGEML_OK;
  dim3 block(128);
  dim3 grid((unsigned)((H / 8 + block.x - 1) / block.x), (unsigned)T_);
  SB_CHECK_ARG(T_ <= 65535 * 64, "combine: too many tokens");
  if (grid.y > 65535) {
    // split tokens over several launches
    for (int t0 = 0; t0 < T_; t0 += 65535) {
      const int nt = std::min(65535, T_ - t0);
      dim3 g2(grid.x, (unsigned)nt);
      if (dtype_bf16)
        (combine_kernel<bf16><<<g2, block, 0, stream>>>(static_cast<const bf16*>(y), pair_row + (int64_t)t0 * kk, nt,
                                                        kk, H, static_cast<bf16*>(out) + (int64_t)t0 * H, T_dev, t0),
         ::sb::count_launch());
      else
        (combine_kernel<f16><<<g2, block, 0, stream>>>(static_cast<const f16*>(y), pair_row + (int64_t)t0 * kk, nt,
                                                       kk, H, static_cast<f16*>(out) + (int64_t)t0 * H, T_dev, t0),
         ::sb::count_launch());
    }
  } else if (dtype_bf16) {
    SB_CUDA_CHECK(launch_kernel(combine_kernel<bf16>, grid, block, 0, stream, pdl, static_cast<const bf16*>(y), pair_row,
                                T_, kk, H, static_cast<bf16*>(out), T_dev, 0));
    ::sb::count_launch();
  } else {
    SB_CUDA_CHECK(launch_kernel(combine_kernel<f16>, grid, block, 0, stream, pdl, static_cast<const f16*>(y), pair_row,
                                T_, kk, H, static_cast<f16*>(out), T_dev, 0));
    ::sb::count_launch();
  }
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

int launch_validate_tenants(const int32_t* in, int64_t n, int n_tenants, int32_t* out, int32_t* status,
                            cudaStream_t stream, bool pdl) {
  if (n == 0) return STAGEML_OK;
  SB_CUDA_CHECK(launch_kernel(validate_tenants_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, pdl, in,
                              n, n_tenants, out, status));
  ::sb::count_launch();
  SB_CUDA_CHECK(cudaGetLastError());
  return STAGEML_OK;
}

}  // namespace sb
